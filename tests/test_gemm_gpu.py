"""The tcgen05 projection GEMM (yuf_gemm_bf16) against a float64 product of the
same bf16 operands.  Shapes with at least 512 rows and columns and enough 256 x
256 tiles run on CTA pairs (cta_group::2), the others on single CTAs; both are
covered.  Compared through the C ABI, at the engine's shapes (configs 1, 3, 4
and 5: R/K/V, low-rank, output, ROSA, FFN, LM head; prefill rows and decode
batches) and at ragged ones (rows, columns and K that are not tile multiples,
unaligned output strides).

Tolerance: the products of bf16 values are exact in fp32 and only the
accumulation order differs from the float64 reference, so fp32 outputs are held
to |got - want| <= 1e-3 sqrt(K) + 1e-3 |want|; bf16 outputs add the output
rounding (rel 2^-8).
"""

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from yufmusicgen_b200 import _lib  # noqa: E402

F32, BF16, BF16_TANH0, SILU_GATE = 0, 1, 2, 3
DEV = "cuda:0"


def gemm(A, lda, a_brows, W, w_brows, C, ldc, c_bstride, M, N, K, batch, epi, acc=0, n_out=0):
    lib = _lib.load()
    st = lib.yuf_gemm_bf16(A.data_ptr(), lda, a_brows, W.data_ptr(), w_brows, C.data_ptr(), ldc, c_bstride,
                           M, N, K, batch, epi, acc, n_out, torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.yuf_last_error().decode()


def rnd(*shape, seed=0, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).to(DEV)


def ref(A, W):
    return A.double() @ W.double().T


def check(got, want, K, bf16=False):
    g, w = got.double().cpu().numpy(), want.double().cpu().numpy()
    rtol = 1e-3 + (2.0 ** -8 if bf16 else 0.0)
    np.testing.assert_allclose(g, w, rtol=rtol, atol=1e-3 * math.sqrt(K))


SHAPES = [  # (M, N, K, batch): engine projections at config 3 / 4 / 5 / 1 sizes, then ragged
    (4096, 640, 640, 3), (4096, 640, 64, 3), (4096, 384, 640, 1), (4096, 640, 128, 1),
    (4096, 640, 2560, 1), (256, 640, 640, 3), (256, 20000, 640, 1), (8192, 1024, 1024, 1),
    (512, 128, 128, 3), (512, 512, 32, 1),
    (1, 64, 32, 1), (100, 100, 40, 1), (129, 200, 72, 2), (300, 1000, 1024, 1), (777, 96, 136, 3),
    (3000, 1300, 200, 3), (2048, 2048, 4096, 1),  # CTA-pair kernel with ragged edges; long K
    (4096, 600, 256, 1),  # 160-column tiles, the last one 120 wide
]


@pytest.mark.parametrize("M,N,K,batch", SHAPES)
def test_gemm_fp32_output_batched(M, N, K, batch):
    A = rnd(batch * M, K, seed=M + K)
    W = rnd(batch * N, K, seed=N + 7, scale=0.05)
    C = torch.full((batch * M, N), float("nan"), device=DEV)
    gemm(A, K, M, W, N, C, N, M * N, M, N, K, batch, F32)
    want = torch.cat([ref(A[z * M:(z + 1) * M], W[z * N:(z + 1) * N]) for z in range(batch)])
    check(C, want, K)


@pytest.mark.parametrize("M,N,K", [(4096, 640, 640), (4096, 640, 2560), (256, 640, 128), (33, 100, 64),
                                   (4096, 1280, 640)])
def test_gemm_accumulates_into_the_residual(M, N, K):
    A = rnd(M, K, seed=1)
    W = rnd(N, K, seed=2, scale=0.05)
    x = torch.randn(M, N, device=DEV)
    C = x.clone()
    gemm(A, K, 0, W, 0, C, N, 0, M, N, K, 1, F32, acc=1)
    check(C, x.double() + ref(A, W), K)


@pytest.mark.parametrize("M,lr,K", [(4096, 64, 640), (256, 64, 640), (512, 32, 128), (50, 96, 1024)])
def test_gemm_bf16_output_with_tanh_on_the_first_batch(M, lr, K):
    A = rnd(3 * M, K, seed=3)
    W = rnd(3 * lr, K, seed=4, scale=0.05)
    C = torch.empty(3 * M, lr, dtype=torch.bfloat16, device=DEV)
    gemm(A, K, M, W, lr, C, lr, M * lr, M, lr, K, 3, BF16_TANH0)
    want = torch.cat([ref(A[z * M:(z + 1) * M], W[z * lr:(z + 1) * lr]) for z in range(3)])
    plain = want.clone()
    want[:M] = torch.tanh(want[:M])
    check(C, want, K, bf16=True)
    C2 = torch.empty_like(C)
    gemm(A, K, M, W, lr, C2, lr, M * lr, M, lr, K, 3, BF16)
    check(C2, plain, K, bf16=True)


def pack_silu_gate(Win, Wg):
    """Rows in groups of 128: 64 rows of the input projection, the same 64 rows of
    the gate (hidden width padded to a multiple of 64 with zero rows)."""
    F, K = Win.shape
    Fp = (F + 63) // 64 * 64
    pad = lambda w: torch.cat([w, torch.zeros(Fp - F, K, dtype=w.dtype, device=w.device)])
    a, b = pad(Win).view(Fp // 64, 64, K), pad(Wg).view(Fp // 64, 64, K)
    return torch.stack([a, b], 1).reshape(2 * Fp, K).contiguous()


@pytest.mark.parametrize("M,d", [(4096, 640), (256, 640), (8192, 1024), (70, 128), (5, 40)])
def test_gemm_silu_gate_epilogue(M, d):
    F = 4 * d
    A = rnd(M, d, seed=5)
    Win, Wg = rnd(F, d, seed=6, scale=0.05), rnd(F, d, seed=7, scale=0.05)
    Wp = pack_silu_gate(Win, Wg)
    H = torch.empty(M, F, dtype=torch.bfloat16, device=DEV)
    gemm(A, d, 0, Wp, 0, H, F, 0, M, Wp.shape[0], d, 1, SILU_GATE, n_out=F)
    hin, hg = ref(A, Win), ref(A, Wg)
    check(H, hin * torch.sigmoid(hin) * hg, d, bf16=True)


def test_gemm_strided_rows_and_unaligned_output():
    """The LM head of the last token: A rows T*d apart (lda = T*d), and an output
    whose row stride is odd (scalar stores)."""
    B, T, d, V = 3, 37, 640, 1001
    Hn = rnd(B * T, d, seed=8)
    E = rnd(V, d, seed=9, scale=0.05)
    last = Hn.view(B, T, d)[:, -1]
    C = torch.zeros(B, V + 2, device=DEV)
    gemm(Hn[T - 1:], T * d, 0, E, 0, C, V + 2, 0, B, V, d, 1, F32)
    check(C[:, :V], ref(last, E), d)
    assert torch.all(C[:, V:] == 0)  # nothing written past N


def test_gemm_rejects_unaligned_operands():
    lib = _lib.load()
    A = rnd(16, 40)
    W = rnd(16, 40)
    C = torch.empty(16, 16, device=DEV)
    s = torch.cuda.current_stream().cuda_stream
    # K = 36 is not a multiple of 8: W rows are not 16-byte aligned
    assert lib.yuf_gemm_bf16(A.data_ptr(), 40, 0, W.data_ptr(), 0, C.data_ptr(), 16, 0, 16, 16, 36, 1,
                             F32, 0, 0, s) == 1
    assert lib.yuf_gemm_bf16(A.data_ptr(), 40, 0, W.data_ptr(), 0, C.data_ptr(), 16, 0, 16, 16, 40, 1,
                             BF16, 1, 0, s) == 1  # accumulate needs the fp32 epilogue
    torch.cuda.synchronize()
    assert lib.yuf_sync_check(s) == 0


# ---- fp32 operands at fp32 accuracy (3xTF32, yuf_gemm_tf32x3) -------------
# Against a float64 product of the fp32 operands: the three tf32 products keep
# each product to about 2^-20, so |got - want| <= 4e-6 sqrt(K) max|A| max|W| +
# 1e-5 |want| (an emulation of the scheme errs by 1e-6 .. 5e-6 absolute at
# these shapes; dropping either low part would err by 2e-3 and fail).
F32_TANH0, SILU_GATE_F32 = 4, 5


def split32(W):
    w = np.ascontiguousarray(W.detach().cpu().numpy(), np.float32)
    hi, lo = np.empty_like(w), np.empty_like(w)
    assert _lib.load().yuf_tf32_split(w.ctypes.data, w.size, hi.ctypes.data, lo.ctypes.data) == 0
    return torch.from_numpy(hi).to(DEV), torch.from_numpy(lo).to(DEV)


def gemm32(A, lda, a_brows, Wh, Wl, w_brows, C, ldc, c_bstride, M, N, K, batch, epi, acc=0, n_out=0):
    lib = _lib.load()
    st = lib.yuf_gemm_tf32x3(A.data_ptr(), lda, a_brows, Wh.data_ptr(), Wl.data_ptr(), w_brows, C.data_ptr(),
                             ldc, c_bstride, M, N, K, batch, epi, acc, n_out,
                             torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.yuf_last_error().decode()


def check32(got, want, K, scale):
    np.testing.assert_allclose(got.double().cpu().numpy(), want.double().cpu().numpy(), rtol=1e-5,
                               atol=4e-6 * math.sqrt(K) * scale)


SHAPES32 = [(4096, 640, 640, 3), (4096, 640, 2560, 1), (256, 640, 640, 3), (256, 20000, 640, 1), (256, 640, 2560, 1),
            (1, 64, 32, 1), (100, 100, 40, 1), (129, 200, 72, 2), (777, 96, 136, 3), (2, 384, 640, 1)]


@pytest.mark.parametrize("M,N,K,batch", SHAPES32)
def test_gemm_tf32x3_matches_fp32(M, N, K, batch):
    g = torch.Generator().manual_seed(M + N + K)
    A = torch.randn(batch * M, K, generator=g).to(DEV)
    W = (torch.randn(batch * N, K, generator=g) * 0.05).to(DEV)
    Wh, Wl = split32(W)
    C = torch.full((batch * M, N), float("nan"), device=DEV)
    gemm32(A, K, M, Wh, Wl, N, C, N, M * N, M, N, K, batch, F32)
    want = torch.cat([ref(A[z * M:(z + 1) * M], W[z * N:(z + 1) * N]) for z in range(batch)])
    check32(C, want, K, float(A.abs().max() * W.abs().max()))


def test_gemm_tf32x3_residual_tanh_and_silu_gate():
    g = torch.Generator().manual_seed(5)
    M, d, lr = 300, 640, 64
    A = torch.randn(M, d, generator=g).to(DEV)
    W = (torch.randn(d, d, generator=g) * 0.05).to(DEV)
    Wh, Wl = split32(W)
    x = torch.randn(M, d, generator=g).to(DEV)
    C = x.clone()
    gemm32(A, d, 0, Wh, Wl, 0, C, d, 0, M, d, d, 1, F32, acc=1)
    check32(C, x.double() + ref(A, W), d, float(A.abs().max() * W.abs().max()))
    # low-rank first stage: three batches, tanh on the first
    A3 = torch.randn(3 * M, d, generator=g).to(DEV)
    L1 = (torch.randn(3 * lr, d, generator=g) * 0.05).to(DEV)
    Lh, Ll = split32(L1)
    C3 = torch.empty(3 * M, lr, device=DEV)
    gemm32(A3, d, M, Lh, Ll, lr, C3, lr, M * lr, M, lr, d, 3, F32_TANH0)
    want = torch.cat([ref(A3[z * M:(z + 1) * M], L1[z * lr:(z + 1) * lr]) for z in range(3)])
    want[:M] = torch.tanh(want[:M])
    check32(C3, want, d, float(A3.abs().max() * L1.abs().max()))
    # FFN: SiLU(in) * gate with the packed in/gate weight, fp32 out
    F = 4 * d
    Win, Wg = (torch.randn(F, d, generator=g) * 0.05).to(DEV), (torch.randn(F, d, generator=g) * 0.05).to(DEV)
    Wp = pack_silu_gate(Win, Wg)
    Ph, Pl = split32(Wp)
    H = torch.empty(M, F, device=DEV)
    gemm32(A, d, 0, Ph, Pl, 0, H, F, 0, M, Wp.shape[0], d, 1, SILU_GATE_F32, n_out=F)
    hin, hg = ref(A, Win), ref(A, Wg)
    np.testing.assert_allclose(H.double().cpu().numpy(), (hin * torch.sigmoid(hin) * hg).cpu().numpy(),
                               rtol=1e-4, atol=1e-4)
