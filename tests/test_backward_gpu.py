"""GPU parity of the training backward ops (yuf_wkv7_backward, yuf_rosa_backward)
against gradients torch autograd computes through the reference's own CPU
recurrences (tests/golden/grads_cases.npz) and against the numpy reverse-mode
oracle (oracle/grads.py) at larger sizes.

Tolerance: |got - want| <= 2e-4 * max|want| + 1e-4 * |want| per gradient
(gradients accumulate over T, so the absolute part scales with the largest
magnitude of each tensor).
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle.grads import rosa_backward as np_rosa_bwd, wkv7_backward as np_wkv_bwd  # noqa: E402
from yufmusicgen_b200 import cuda_ops, rosa_cuda  # noqa: E402
from yufmusicgen_b200.workloads import rosa_op_inputs, wkv_op_inputs  # noqa: E402

DEV = "cuda:0"


def cu(x, grad=False):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(DEV)
    return t.requires_grad_(True) if grad else t


def close(got, want, rel=2e-4):
    got = got.detach().cpu().numpy() if hasattr(got, "detach") else got
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=rel * float(np.abs(want).max()))


@pytest.mark.parametrize("case", ["w_n40", "w_n16", "w_n64", "w_n32_t20"])
def test_rwkv7_cuda_autograd_matches_reference_autograd(golden, case):
    g = golden("grads_cases.npz")
    xs = [cu(g[f"{case}.{k}"], grad=True) for k in "rwkvab"]
    y, _ = cuda_ops.rwkv7_cuda(*xs)
    close(y, g[f"{case}.y"])
    (y * cu(g[f"{case}.dy"])).sum().backward()
    for k, x in zip("rwkvab", xs):
        close(x.grad, g[f"{case}.d{k}"])


@pytest.mark.parametrize("B,T,H,N", [(2, 128, 3, 40), (1, 64, 2, 128), (2, 96, 2, 96), (3, 48, 2, 48)])
def test_wkv7_torch_op_backward_vs_oracle(B, T, H, N):
    """torch.ops.yufmusicgen_rwkv7.forward/backward with the reference's
    preallocated buffers (rwkv7_clampw.cpp:18-63), several chunks per chain."""
    import yufmusicgen_b200.torch_ops  # noqa: F401

    ins = wkv_op_inputs(B, T, H, N, seed=B * 100 + T + N)
    dy = np.random.default_rng(T + N).standard_normal((B, T, H, N), dtype=np.float32)
    t = [cu(ins[k]) for k in "rwkvab"]
    y = torch.empty_like(t[0])
    states = torch.empty(B, H, T // 16, N, N, device=DEV)
    sa = torch.empty_like(t[0])
    torch.ops.yufmusicgen_rwkv7.forward(*t, y, states, sa)
    grads = [torch.empty_like(t[0]) for _ in range(6)]
    torch.ops.yufmusicgen_rwkv7.backward(*t, cu(dy), states, sa, *grads)
    want = np_wkv_bwd(*(ins[k] for k in "rwkvab"), dy)
    for got, w in zip(grads, want):
        close(got, w)


@pytest.mark.parametrize("case", ["r_r32", "r_r128", "r_r256"])
def test_rosa_householder_scan_autograd_matches_reference_autograd(golden, case):
    g = golden("grads_cases.npz")
    keys = ("cand", "write", "decay", "direction", "m0")
    xs = {k: cu(g[f"{case}.{k}"], grad=True) for k in keys}
    gate = torch.zeros_like(xs["cand"]).requires_grad_(True)
    read, _ = rosa_cuda.rosa_householder_scan(xs["cand"], xs["write"], gate, xs["decay"],
                                              xs["direction"], xs["m0"])
    close(read, g[f"{case}.read"])
    (read * cu(g[f"{case}.dq"])).sum().backward()
    for k in keys:
        close(xs[k].grad, g[f"{case}.d{k}"])
    assert float(gate.grad.abs().max()) == 0.0  # the ungated read does not depend on read_raw


def _rosa_saved(ins):
    """The forward op's saved tensors, built on the host (any R)."""
    cand, write, decay, d, m0 = (ins[k] for k in ("cand", "write", "decay", "direction", "m0"))
    B, T, R = cand.shape
    c, wg = np.tanh(cand), 1.0 / (1.0 + np.exp(-write))
    mem = np.empty((B, T + 1, R), np.float32)
    mem[:, 0] = m0
    m = m0.astype(np.float64)
    for t in range(T):
        h = m - 2.0 * (m @ d)[:, None] * d
        m = decay * h + wg[:, t] * c[:, t]
        mem[:, t + 1] = m
    return (c.astype(np.float32), wg.astype(np.float32),
            np.broadcast_to(decay, (B, T, R)).astype(np.float32), mem)


@pytest.mark.parametrize("B,T,R", [(3, 9, 12), (2, 300, 100), (4, 129, 512), (1, 1, 32)])
def test_rosa_backward_any_R_vs_oracle(B, T, R):
    ins = rosa_op_inputs(B, T, R, seed=B + T + R, with_state=True)
    dq = np.random.default_rng(R + T).standard_normal((B, T, R), dtype=np.float32)
    cs, ws, ds, ms = _rosa_saved(ins)
    d_cand, d_write, d_raw, d_decay, d_dir, d_mem = rosa_cuda.rosa_backward(
        cu(cs), cu(ws), cu(cs), cu(ws), cu(ds), cu(ms), cu(ins["direction"]), cu(ms[:, -1]), cu(dq))
    want = np_rosa_bwd(*(ins[k] for k in ("cand", "write", "decay", "direction", "m0")), dq)
    for got, w in zip((d_cand, d_write, d_decay, d_dir, d_mem), want):
        close(got, w)
    assert float(d_raw.abs().max()) == 0.0


def test_rosa_torch_op_backward_matches_autograd_path():
    """torch.ops.yufmusicgen_rosa.forward/backward with the reference's buffers
    (rosa_householder.cpp:24-83) equal the autograd path."""
    import yufmusicgen_b200.torch_ops  # noqa: F401

    B, T, R = 2, 40, 64
    ins = rosa_op_inputs(B, T, R, seed=77, with_state=True)
    dq = cu(np.random.default_rng(78).standard_normal((B, T, R), dtype=np.float32))
    a = [cu(ins[k]) for k in ("cand", "write", "read_gate", "decay", "direction", "m0")]
    read_out = torch.empty(B, T, R, device=DEV)
    memory_out = torch.empty(B, R, device=DEV)
    saved = [torch.empty(B, T, R, device=DEV) for _ in range(5)]
    mem_saved = torch.empty(B, T + 1, R, device=DEV)
    torch.ops.yufmusicgen_rosa.forward(*a, read_out, memory_out, *saved, mem_saved)
    outs = [torch.empty(B, T, R, device=DEV) for _ in range(4)]
    d_dir = torch.empty(B, R, device=DEV)
    d_mem = torch.empty(B, R, device=DEV)
    ws = torch.empty(B, T, 5 * R, device=DEV)
    torch.ops.yufmusicgen_rosa.backward(*saved, mem_saved, a[4], memory_out, dq, *outs, d_dir, d_mem, ws)
    xs = [x.clone().requires_grad_(True) for x in a]
    read, _ = rosa_cuda.rosa_householder_scan(*xs)
    (read * dq).sum().backward()
    close(outs[0], xs[0].grad.cpu().numpy())
    close(outs[1], xs[1].grad.cpu().numpy())
    close(outs[3].sum((0, 1)), xs[3].grad.cpu().numpy())
    close(d_dir.sum(0), xs[4].grad.cpu().numpy())
    close(d_mem, xs[5].grad.cpu().numpy())
