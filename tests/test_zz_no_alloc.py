"""yuf_step_static: the decode step for callers that may not allocate device
memory while they run (a real-time audio callback, a component with a fixed
memory budget).  It must give the same logits and leave the same state as the
ordinary yuf_step, call after call, allocate nothing on a model that has never
run a prefill, and refuse exactly the batches its fixed scratch cannot hold.

The file name sorts last so a run that stops at the first failure has already
run every other test; it also passes on its own in a fresh process.
Tolerance: the fp32 path's |got - want| <= 1e-3 + 1e-4 |want| (both calls run
the same kernels in the same precision, so bf16-weight mode is held to it too).
"""

import re

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from yufmusicgen_b200 import _lib  # noqa: E402
from yufmusicgen_b200 import config as C  # noqa: E402
from yufmusicgen_b200.engine import Engine  # noqa: E402
from yufmusicgen_b200.weights import init_weights  # noqa: E402
from yufmusicgen_b200.workloads import tiny_ids  # noqa: E402

RTOL, ATOL = 1e-4, 1e-3


def _step_static(eng, ids, slot0, out):
    lib = _lib.load()
    return lib.yuf_step_static(eng._h, ids.data_ptr(), ids.numel(), slot0, out.data_ptr(),
                               torch.cuda.current_stream().cuda_stream)


def _max_batch(eng):
    """The largest batch the fixed scratch holds, from the refusal message."""
    ids = torch.zeros(1 << 20, dtype=torch.int32, device="cuda")
    out = torch.empty(1, device="cuda")
    assert _step_static(eng, ids, 0, out) == 1  # YUF_ERR_INVALID_ARGUMENT, before any launch
    msg = _lib.load().yuf_last_error().decode()
    m = re.search(r"at most (\d+) sequences", msg)
    assert m and "scratch" in msg, msg
    return int(m.group(1))


def _states_equal(eng, layers, a0, b0, n):
    for layer in range(layers):
        a = eng.export_state(layer, a0, n)
        b = eng.export_state(layer, b0, n)
        for key in ("prev", "S", "m"):
            np.testing.assert_allclose(b[key].cpu().numpy(), a[key].cpu().numpy(), rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_step_static_matches_step_on_consecutive_calls(precision):
    cfg = C.ModelConfig(**C.TINY)
    eng = Engine(cfg, init_weights(cfg, 0, "perturbed"), precision=precision, n_slots=4)
    prompt = torch.as_tensor(tiny_ids(2, 20, seed=5), dtype=torch.int32, device="cuda")
    eng.prefill(prompt, slot0=0)  # slots 0-1: ordinary step
    eng.prefill(prompt, slot0=2)  # slots 2-3: allocation-free step, same starting state
    tok = torch.tensor([7, 301], dtype=torch.int32, device="cuda")
    for _ in range(2):  # two calls in a row: the scratch keeps the previous call's contents
        want = eng.step(tok, slot0=0)
        got = torch.empty_like(want)
        st = _step_static(eng, tok, 2, got)
        assert st == 0, _lib.load().yuf_last_error().decode()
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=RTOL, atol=ATOL)
        tok = torch.argmax(want, dim=-1).to(torch.int32)
    _states_equal(eng, cfg.n_layers, 0, 2, 2)
    eng.sync_check()
    eng.close()


def test_step_static_allocates_nothing_on_a_fresh_model():
    """A model that only has its state slots (no prefill, so no workspace):
    the device's free memory is the same before and after two static steps."""
    cfg = C.ModelConfig(**C.TINY)
    w = init_weights(cfg, 0, "perturbed")
    # load every kernel module once (lazy loading places module code in device memory)
    warm = Engine(cfg, w, n_slots=2)
    tok = torch.tensor([7, 301], dtype=torch.int32, device="cuda")
    out = torch.empty(2, cfg.vocab_size, device="cuda")
    assert _step_static(warm, tok, 0, out) == 0
    warm.step(tok, slot0=0)
    torch.cuda.synchronize()
    warm.close()
    eng = Engine(cfg, w, n_slots=4)
    got = [torch.empty(2, cfg.vocab_size, device="cuda") for _ in range(2)]
    ids = [tok, torch.tensor([11, 400], dtype=torch.int32, device="cuda")]
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for i in range(2):
        assert _step_static(eng, ids[i], 2, got[i]) == 0, _lib.load().yuf_last_error().decode()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    for i in range(2):  # the ordinary step from the same (zero) state on slots 0-1
        want = eng.step(ids[i], slot0=0)
        np.testing.assert_allclose(got[i].cpu().numpy(), want.cpu().numpy(), rtol=RTOL, atol=ATOL)
    _states_equal(eng, cfg.n_layers, 0, 2, 2)
    eng.close()


def test_step_static_runs_the_largest_batch_and_refuses_one_more():
    cfg = C.ModelConfig(**C.TINY)
    probe = Engine(cfg, init_weights(cfg, 0, "perturbed"), n_slots=1)
    bmax = _max_batch(probe)
    probe.close()
    assert bmax >= 2
    eng = Engine(cfg, init_weights(cfg, 0, "perturbed"), n_slots=2 * bmax + 1)
    g = torch.Generator().manual_seed(3)
    tok = torch.randint(0, cfg.vocab_size, (bmax,), generator=g, dtype=torch.int32).cuda()
    got = torch.empty(bmax, cfg.vocab_size, device="cuda")
    assert _step_static(eng, tok, bmax, got) == 0, _lib.load().yuf_last_error().decode()
    want = eng.step(tok, slot0=0)
    torch.cuda.synchronize()
    np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=RTOL, atol=ATOL)
    _states_equal(eng, cfg.n_layers, 0, bmax, bmax)
    one_more = torch.zeros(bmax + 1, dtype=torch.int32, device="cuda")
    out = torch.empty(bmax + 1, cfg.vocab_size, device="cuda")
    assert _step_static(eng, one_more, 0, out) == 1
    assert f"at most {bmax} sequences" in _lib.load().yuf_last_error().decode()
    eng.close()
