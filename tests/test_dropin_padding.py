"""The reference op wrapper's own padding path, through this library's ops.

``yufmusicgen/cuda_ops.py:160-186`` (``_pad_inputs``) pads T to a multiple of
16 with zero r/k/v/a/b and w_raw = -80, hands the padded tensors to
``torch.ops.yufmusicgen_rwkv7.forward`` with preallocated outputs, then keeps
``output[:, :T]`` and the last checkpoint transposed as the final state
(cuda_ops.py:211-232).  ``tests/golden/dropin_pad_cases.npz`` holds what that
wrapper produced (``make_golden.py dropin``) together with the reference CPU
recurrence's y and final state for the unpadded inputs.

* CPU: ``cuda_ops._pad16`` pads exactly as the reference wrapper did.
* GPU: the wrapper's padded tensors through ``torch.ops.yufmusicgen_rwkv7.forward``
  and the wrapper's post-processing give the reference's outputs; so does the
  drop-in ``cuda_ops.rwkv7_cuda`` on the unpadded inputs.
  Tolerance: |got - want| <= 1e-3 + 1e-4 |want|.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

CASES = ["n40_t21", "n64_t5", "n16_t37"]
ARGS = ("r", "w", "k", "v", "a", "b")


@pytest.mark.parametrize("case", CASES)
def test_pad16_matches_the_reference_wrapper(golden, case):
    from yufmusicgen_b200 import cuda_ops

    g = golden("dropin_pad_cases.npz")
    ins = [torch.from_numpy(g[f"{case}.{k}"]) for k in ARGS]
    padded, length = cuda_ops._pad16(*ins)
    assert length == int(g[f"{case}.length"])
    for k, x in zip(ARGS, padded):
        np.testing.assert_array_equal(x.numpy(), g[f"{case}.{k}_padded"])


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_reference_wrapper_path_through_the_registered_op(golden, case):
    import yufmusicgen_b200.torch_ops  # noqa: F401  (registers torch.ops.yufmusicgen_rwkv7)

    g = golden("dropin_pad_cases.npz")
    p = [torch.from_numpy(g[f"{case}.{k}_padded"]).cuda() for k in ARGS]
    length = int(g[f"{case}.length"])
    B, Tp, H, N = p[0].shape
    output = torch.empty_like(p[3])
    states = torch.empty(B, H, Tp // 16, N, N, device="cuda", dtype=torch.float32)
    sa = torch.empty_like(p[0])
    torch.ops.yufmusicgen_rwkv7.forward(*p, output, states, sa)
    torch.cuda.synchronize()
    y = output[:, :length].cpu().numpy()
    final_state = states[:, :, -1].transpose(-1, -2).contiguous().cpu().numpy()
    np.testing.assert_allclose(y, g[f"{case}.y"], rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(final_state, g[f"{case}.sT"], rtol=1e-4, atol=1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_dropin_rwkv7_cuda_on_unpadded_inputs(golden, case):
    from yufmusicgen_b200 import cuda_ops

    g = golden("dropin_pad_cases.npz")
    ins = [torch.from_numpy(g[f"{case}.{k}"]).cuda().requires_grad_(True) for k in ARGS]
    y, s = cuda_ops.rwkv7_cuda(*ins)  # the differentiable path pads as the reference does
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.detach().cpu().numpy(), g[f"{case}.y"], rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(s.detach().cpu().numpy(), g[f"{case}.sT"], rtol=1e-4, atol=1e-3)
