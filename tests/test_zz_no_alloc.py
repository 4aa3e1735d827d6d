"""yuf_step_static: the decode step for callers that may not allocate device
memory while they run (a real-time audio callback, a component with a fixed
memory budget).  It must give the same logits and leave the same state as the
ordinary yuf_step, call after call, and refuse batches its fixed scratch
cannot hold.

The file name sorts last so a run that stops at the first failure has already
run every other test; it also passes on its own in a fresh process.
Tolerance: the fp32 path's |got - want| <= 1e-3 + 1e-4 |want|.
"""

import ctypes

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


def test_step_static_matches_step_on_consecutive_calls():
    cfg = C.ModelConfig(**C.TINY)
    eng = Engine(cfg, init_weights(cfg, 0, "perturbed"), n_slots=4)
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
    for layer in range(cfg.n_layers):
        a = eng.export_state(layer, 0, 2)
        b = eng.export_state(layer, 2, 2)
        for key in ("prev", "S", "m"):
            np.testing.assert_allclose(b[key].cpu().numpy(), a[key].cpu().numpy(), rtol=RTOL, atol=ATOL)
    eng.sync_check()
    eng.close()


def test_step_static_rejects_batches_beyond_its_scratch():
    cfg = C.ModelConfig(**C.TINY)
    eng = Engine(cfg, init_weights(cfg, 0, "perturbed"), n_slots=2)
    ids = torch.zeros(100000, dtype=torch.int32, device="cuda")
    out = torch.empty(1, device="cuda")
    st = _step_static(eng, ids, 0, out)
    assert st == 1  # YUF_ERR_INVALID_ARGUMENT, before any launch
    msg = _lib.load().yuf_last_error().decode()
    assert "scratch" in msg and "at most" in msg
    eng.close()
