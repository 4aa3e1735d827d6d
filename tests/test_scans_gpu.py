"""GPU parity of the WKV-7 and ROSA scan kernels against the CPU oracle.

Tolerance (fp32 path): |got - want| <= 1e-3 + 1e-4 * |want| element-wise
(``max-abs 1e-3 / rel 1e-4``), checked with numpy.testing.assert_allclose.
Small cases also compare against the reference's own outputs
(tests/golden/*.npz); full benchmark sizes compare against the C oracle.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import cref  # noqa: E402
from oracle.scans import rosa_scan as np_rosa, rosa_scan_ungated, wkv7_scan as np_wkv  # noqa: E402
from yufmusicgen_b200 import cuda_ops, rosa_cuda  # noqa: E402
from yufmusicgen_b200.workloads import rosa_op_inputs, wkv_op_inputs  # noqa: E402

RTOL, ATOL = 1e-4, 1e-3
DEV = "cuda:0"


def cu(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def close(got, want, rtol=RTOL, atol=ATOL):
    np.testing.assert_allclose(got.detach().cpu().numpy() if hasattr(got, "cpu") else got, want,
                               rtol=rtol, atol=atol)


WKV_CASES = ["n40_state", "n32_zero", "n64_state", "n16_state", "n40_t1"]


ALGOS = [cuda_ops.ALGO_SEQUENTIAL, cuda_ops.ALGO_CHUNKED, cuda_ops.ALGO_ROWS, cuda_ops.ALGO_CHUNKED_TC]


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("case", WKV_CASES)
def test_wkv7_matches_reference_golden(golden, case, algo):
    g = golden("wkv7_cases.npz")
    ins = [cu(g[f"{case}.{k}"]) for k in ("r", "w", "k", "v", "a", "b")]
    y, s = cuda_ops.wkv7_forward(*ins, state=cu(g[f"{case}.s0"]), algo=algo)
    torch.cuda.synchronize()
    close(y, g[f"{case}.y"])
    close(s, g[f"{case}.sT"])


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("T", [0, 1, 15, 16, 17, 63, 200])
@pytest.mark.parametrize("N", [16, 32, 40, 48, 64, 96, 128])
def test_wkv7_ragged_T_and_head_sizes(T, N, algo):
    ins = wkv_op_inputs(2, T, 3, N, seed=100 + T + N, with_state=True)
    if algo == cuda_ops.ALGO_CHUNKED_TC and N > 64 and T > 1:
        with pytest.raises(RuntimeError, match="no kernel"):
            cuda_ops.wkv7_forward(*(cu(ins[k]) for k in "rwkvab"), state=cu(ins["s0"]), algo=algo)
        return
    y, s = cuda_ops.wkv7_forward(*(cu(ins[k]) for k in "rwkvab"), state=cu(ins["s0"]), algo=algo)
    yr, sr = np_wkv(*(ins[k] for k in "rwkvab"), ins["s0"])
    close(y, yr)
    close(s, sr)


@pytest.mark.parametrize("algo", ALGOS)
def test_wkv7_full_config2_vs_c_oracle(algo):
    """The benchmark workload itself: B8 T2048 H16 N40, zero state."""
    ins = wkv_op_inputs(8, 2048, 16, 40, seed=0)
    y, s = cuda_ops.wkv7_forward(*(cu(ins[k]) for k in "rwkvab"), algo=algo)
    yr, sr = cref.wkv7_scan(*(ins[k] for k in "rwkvab"))
    close(y, yr)
    close(s, sr)


def test_wkv7_decode_steps_equal_prefill():
    """Prefill 100 tokens then 20 single-token steps == one 120-token scan."""
    ins = wkv_op_inputs(4, 120, 16, 40, seed=5, with_state=True)
    t = {k: cu(ins[k]) for k in "rwkvab"}
    y_full, s_full = cuda_ops.wkv7_forward(*(t[k] for k in "rwkvab"), state=cu(ins["s0"]))
    state = cu(ins["s0"]).clone()
    y_pre, state = cuda_ops.wkv7_forward(*(t[k][:, :100].contiguous() for k in "rwkvab"), state=state)
    ys = [y_pre]
    for i in range(100, 120):
        yi, _ = cuda_ops.wkv7_forward(*(t[k][:, i:i + 1].contiguous() for k in "rwkvab"), state=state,
                                      state_out=state)  # in place
        ys.append(yi)
    close(torch.cat(ys, 1), y_full.cpu().numpy(), rtol=1e-5, atol=1e-5)
    close(state, s_full.cpu().numpy(), rtol=1e-5, atol=1e-5)


def test_wkv7_long_head64_state_vs_c_oracle():
    """Config-5 head geometry (N=64) over a long sequence with a carried state."""
    ins = wkv_op_inputs(2, 4096, 16, 64, seed=8, with_state=True)
    y, s = cuda_ops.wkv7_forward(*(cu(ins[k]) for k in "rwkvab"), state=cu(ins["s0"]))
    yr, sr = cref.wkv7_scan(*(ins[k] for k in "rwkvab"), ins["s0"])
    close(y, yr)
    close(s, sr)


def test_wkv7_batched_decode_config4_shape():
    """One decode step of 256 sequences x 16 heads x N40 with a random state."""
    ins = wkv_op_inputs(256, 1, 16, 40, seed=9, with_state=True)
    y, s = cuda_ops.wkv7_forward(*(cu(ins[k]) for k in "rwkvab"), state=cu(ins["s0"]))
    yr, sr = cref.wkv7_scan(*(ins[k] for k in "rwkvab"), ins["s0"])
    close(y, yr)
    close(s, sr)


def test_wkv7_validation_errors_match_reference():
    x = torch.zeros(1, 16, 1, 40, device=DEV)
    with pytest.raises(ValueError):
        cuda_ops.rwkv7_cuda(x[0], x[0], x[0], x[0], x[0], x[0])
    with pytest.raises(TypeError):
        d = x.double()
        cuda_ops.rwkv7_cuda(d, d, d, d, d, d)
    with pytest.raises(ValueError):
        nc = torch.zeros(1, 40, 1, 16, device=DEV).transpose(1, 3)
        cuda_ops.rwkv7_cuda(nc, nc, nc, nc, nc, nc)
    with pytest.raises(ValueError):
        cuda_ops.rwkv7_cuda(x, x, x, x, x, torch.zeros(1, 32, 1, 40, device=DEV))


def _compat_expected(ins):
    """Chunk checkpoints (transposed) and sa from the numpy oracle, step by step."""
    r, w, k, v, a, b = (ins[x] for x in "rwkvab")
    B, T, H, N = r.shape
    S = np.zeros((B, H, N, N), np.float32)
    sa = np.empty((B, T, H, N), np.float32)
    ck = np.empty((B, H, T // 16, N, N), np.float32)
    for t in range(T):
        sa[:, t] = np.einsum("bhj,bhij->bhi", a[:, t], S)
        _, S = np_wkv(r[:, t:t + 1], w[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], a[:, t:t + 1],
                      b[:, t:t + 1], S)
        if (t + 1) % 16 == 0:
            ck[:, :, t // 16] = np.swapaxes(S, -1, -2)
    return ck, sa


def test_torch_op_drop_in_rwkv7_forward():
    """torch.ops.yufmusicgen_rwkv7.forward with the reference's preallocated outputs."""
    import yufmusicgen_b200.torch_ops  # noqa: F401

    ins = wkv_op_inputs(2, 48, 3, 40, seed=21)
    t = [cu(ins[k]) for k in "rwkvab"]
    B, T, H, N = t[0].shape
    y = torch.empty_like(t[0])
    states = torch.empty(B, H, T // 16, N, N, device=DEV)
    sa = torch.empty_like(t[0])
    torch.ops.yufmusicgen_rwkv7.forward(*t, y, states, sa)
    yr, sr = np_wkv(*(ins[k] for k in "rwkvab"))
    ck, sar = _compat_expected(ins)
    close(y, yr)
    close(states, ck)
    close(sa, sar)
    # cuda_ops.py:231's final_state = states[:, :, -1].transpose(-1, -2) is canonical S
    close(states[:, :, -1].transpose(-1, -2), sr)


ROSA_CASES = ["r32_state", "r128_zero", "r256_state", "r12_state", "r128_t1"]


@pytest.mark.parametrize("case", ROSA_CASES)
def test_rosa_matches_reference_golden(golden, case):
    g = golden("rosa_cases.npz")
    args = [cu(g[f"{case}.{k}"]) for k in ("cand", "write", "read_gate", "decay", "direction", "m0")]
    read, m = rosa_cuda.rosa_scan(*args, gated=True)
    close(read, g[f"{case}.read"])
    close(m, g[f"{case}.mT"])
    ung, m2 = rosa_cuda.rosa_householder_scan(*args)
    gate = 1.0 / (1.0 + np.exp(-g[f"{case}.read_gate"]))
    close(ung.cpu().numpy() * gate, g[f"{case}.read"])


@pytest.mark.parametrize("T", [0, 1, 16, 17, 33, 257])
@pytest.mark.parametrize("R", [1, 12, 32, 100, 128, 256, 512])
def test_rosa_ragged(T, R):
    ins = rosa_op_inputs(3, T, R, seed=T * 7 + R, with_state=True)
    args = [cu(ins[k]) for k in ("cand", "write", "read_gate", "decay", "direction", "m0")]
    read, m = rosa_cuda.rosa_scan(*args, gated=True)
    rr, mr = np_rosa(*(ins[k] for k in ("cand", "write", "read_gate", "decay", "direction", "m0")))
    close(read, rr)
    close(m, mr)


def test_rosa_full_config3_size_vs_c_oracle():
    ins = rosa_op_inputs(2, 2048, 128, seed=3)
    args = [cu(ins[k]) for k in ("cand", "write", "read_gate", "decay", "direction", "m0")]
    read, m = rosa_cuda.rosa_scan(*args, gated=True)
    rr, mr = cref.rosa_scan(*(ins[k] for k in ("cand", "write", "read_gate", "decay", "direction", "m0")))
    close(read, rr)
    close(m, mr)


def test_rosa_decay_near_one_is_stable():
    ins = rosa_op_inputs(2, 600, 128, seed=4, with_state=True)
    ins["decay"] = np.full(128, 0.99999, np.float32)
    args = [cu(ins[k]) for k in ("cand", "write", "read_gate", "decay", "direction", "m0")]
    read, m = rosa_cuda.rosa_scan(*args, gated=True)
    rr, mr = cref.rosa_scan(*(ins[k] for k in ("cand", "write", "read_gate", "decay", "direction", "m0")))
    close(read, rr)
    close(m, mr)


def test_torch_op_drop_in_rosa_forward():
    import yufmusicgen_b200.torch_ops  # noqa: F401

    ins = rosa_op_inputs(2, 37, 64, seed=31, with_state=True)
    cand, write, gate, decay, direction, mem = (cu(ins[k]) for k in (
        "cand", "write", "read_gate", "decay", "direction", "m0"))
    B, T, R = cand.shape
    outs = [torch.empty_like(cand), torch.empty_like(mem)] + [torch.empty_like(cand) for _ in range(5)]
    mem_saved = torch.empty(B, T + 1, R, device=DEV)
    torch.ops.yufmusicgen_rosa.forward(cand, write, gate, decay, direction, mem, *outs, mem_saved)
    read_out, memory_out, cs, ws, rs, gs, ds = outs
    ur, mr = rosa_scan_ungated(*(ins[k] for k in ("cand", "write", "read_gate", "decay", "direction", "m0")))
    close(read_out, ur)
    close(memory_out, mr)
    close(rs, ur)
    close(cs, np.tanh(ins["cand"]))
    close(ws, 1 / (1 + np.exp(-ins["write"])))
    close(gs, 1 / (1 + np.exp(-ins["read_gate"])))
    close(ds, np.broadcast_to(ins["decay"], (B, T, R)))
    close(mem_saved[:, 0], ins["m0"])
    close(mem_saved[:, -1], mr)
    _, m_half = np_rosa(*(ins[k][:, :20] if ins[k].ndim == 3 else ins[k]
                          for k in ("cand", "write", "read_gate", "decay", "direction", "m0")))
    close(mem_saved[:, 20], m_half)


PAR_ALGOS = [cuda_ops.ALGO_PARALLEL, cuda_ops.ALGO_PARALLEL_TC]


@pytest.mark.parametrize("algo", PAR_ALGOS)
@pytest.mark.parametrize("T", [256, 300, 1000])
@pytest.mark.parametrize("N", [16, 40, 64, 128])
def test_wkv7_time_parallel_matches_oracle(T, N, algo):
    """Chunks scanned in parallel with carried states (the last chunk ragged);
    the output correction on mma.sync or on the tcgen05 tensor cores."""
    ins = wkv_op_inputs(2, T, 3, N, seed=500 + T + N, with_state=True)
    y, s = cuda_ops.wkv7_forward(*(cu(ins[k]) for k in "rwkvab"), state=cu(ins["s0"]), algo=algo)
    yr, sr = cref.wkv7_scan(*(ins[k] for k in "rwkvab"), ins["s0"])
    close(y, yr)
    close(s, sr)


@pytest.mark.parametrize("B,T,H,N,with_state", [
    (2, 257, 3, 40, False),   # zero start: chunk 0 skips the correction; short last chunk
    (1, 520, 2, 32, True),
    (4, 300, 2, 48, False),
    (2, 1000, 2, 96, True),
    (1, 777, 1, 16, True),
    (40, 256, 16, 40, True),  # many chains: two chunks per sequence
    (16, 1024, 4, 64, True),  # chunks of 208 tokens: two 128-token correction tiles each
    (48, 600, 4, 16, False),  # chunks of 304 tokens: three tiles, the last one ragged
])
@pytest.mark.parametrize("algo", PAR_ALGOS)
def test_wkv7_time_parallel_shapes(B, T, H, N, with_state, algo):
    ins = wkv_op_inputs(B, T, H, N, seed=900 + B + T + N, with_state=with_state)
    s0 = cu(ins["s0"]) if with_state else None
    y, s = cuda_ops.wkv7_forward(*(cu(ins[k]) for k in "rwkvab"), state=s0, algo=algo)
    yr, sr = cref.wkv7_scan(*(ins[k] for k in "rwkvab"), ins["s0"] if with_state else None)
    close(y, yr)
    close(s, sr)


def test_time_parallel_waits_never_expired():
    """The pair kernel's staging barrier waits are bounded; none may have expired."""
    from yufmusicgen_b200 import _lib
    ins = wkv_op_inputs(2, 300, 3, 40, seed=11)
    cuda_ops.wkv7_forward(*(cu(ins[k]) for k in "rwkvab"), algo=cuda_ops.ALGO_PARALLEL)
    torch.cuda.synchronize()
    assert _lib.wait_timeouts() == 0


def test_expired_wait_is_reported_and_the_context_survives():
    """The bounded-wait path end to end: a warp waits (2 ms bound) on a barrier
    nothing arrives at, records the expiry as the scan kernels do, returns; the
    synchronising check reports YUF_ERR_TIMEOUT once, then OK, and the next scan
    on the same context is exact."""
    from yufmusicgen_b200 import _lib
    lib = _lib.load()
    s = torch.cuda.current_stream().cuda_stream
    assert lib.yuf_sync_check(s) == 0
    assert lib.yuf_debug_wait_selftest(2_000_000, s) == 0
    assert lib.yuf_sync_check(s) == 6  # YUF_ERR_TIMEOUT
    assert "expired" in lib.yuf_last_error().decode()
    assert lib.yuf_sync_check(s) == 0  # the count was cleared
    assert lib.yuf_debug_wait_selftest(3_000_000_000, s) == 1  # above the 2 s cap: refused
    ins = wkv_op_inputs(2, 300, 3, 40, seed=12)
    y, st = cuda_ops.wkv7_forward(*(cu(ins[k]) for k in "rwkvab"), algo=cuda_ops.ALGO_PARALLEL)
    yr, sr = cref.wkv7_scan(*(ins[k] for k in "rwkvab"), None)
    close(y, yr)
    close(st, sr)
    assert lib.yuf_sync_check(s) == 0


@pytest.mark.parametrize("B,H,N", [(512, 16, 40), (128, 16, 64), (32, 16, 128), (64, 8, 96)])
def test_wkv7_decode_many_heads_per_cta(B, H, N):
    """Single-token steps with more heads than the decode ring's slots per CTA
    (the slot refill path), in place, then the same step with the state at an
    8-byte offset (the register-prefetch kernel); no bounded wait may expire."""
    from yufmusicgen_b200 import _lib
    ins = wkv_op_inputs(B, 1, H, N, seed=B + N, with_state=True)
    yr, sr = cref.wkv7_scan(*(ins[k] for k in "rwkvab"), ins["s0"])
    t = [cu(ins[k]) for k in "rwkvab"]
    st = cu(ins["s0"])
    y, _ = cuda_ops.wkv7_forward(*t, state=st, state_out=st)
    close(y, yr)
    close(st, sr)
    n = st.numel()
    buf = torch.zeros(n + 2, device=DEV)
    off = buf[2:].view_as(st)  # 8 bytes past a 16-byte boundary
    off.copy_(cu(ins["s0"]))
    y2, _ = cuda_ops.wkv7_forward(*t, state=off, state_out=off)
    close(y2, yr)
    close(off, sr)
    torch.cuda.synchronize()
    assert _lib.wait_timeouts() == 0


@pytest.mark.parametrize("algo", PAR_ALGOS)
def test_wkv7_time_parallel_full_config2_and_inplace_state(algo):
    ins = wkv_op_inputs(8, 2048, 16, 40, seed=0, with_state=True)
    st = cu(ins["s0"])
    y, s = cuda_ops.wkv7_forward(*(cu(ins[k]) for k in "rwkvab"), state=st, state_out=st, algo=algo)
    yr, sr = cref.wkv7_scan(*(ins[k] for k in "rwkvab"), ins["s0"])
    close(y, yr)
    close(st, sr)


@pytest.mark.parametrize("B,T,R", [(1, 1024, 128), (2, 2048, 128), (3, 512, 100), (4, 256, 32), (3, 512, 64), (2, 384, 12),
                                   (2, 512, 256), (8, 1024, 256), (1, 2048, 200), (8, 8192, 256)])
def test_rosa_time_parallel_matches_oracle(B, T, R):
    ins = rosa_op_inputs(B, T, R, seed=B * 1000 + T + R, with_state=True)
    if R >= 128:
        ins["decay"][:8] = 0.9999  # slow channels stress the carried state
    args = [cu(ins[k]) for k in ("cand", "write", "read_gate", "decay", "direction", "m0")]
    read, m = rosa_cuda.rosa_scan(*args, gated=True)
    rr, mr = cref.rosa_scan(*(ins[k] for k in ("cand", "write", "read_gate", "decay", "direction", "m0")))
    close(read, rr)
    close(m, mr)
    ung, _ = rosa_cuda.rosa_householder_scan(*args)
    ur, _ = rosa_scan_ungated(*(ins[k] for k in ("cand", "write", "read_gate", "decay", "direction", "m0")))
    close(ung, ur)
