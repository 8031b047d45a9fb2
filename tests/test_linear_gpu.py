"""GPU checks of the projection GEMMs against float64 products: the
small-batch fp32 kernel (``m3_linear_f32``) over batch sizes, widths and
depths that do and do not fill the 16 x 16 CTA tile and the 128-wide K
slices, strided rows; the split-precision fp32 tensor-core GEMM
(``m3_linear_f32_tc``) that larger fp32 batches take; the bf16 tcgen05 GEMM
(``m3_linear_bf16``); and the size-based dispatch between them and cuBLAS."""

from __future__ import annotations

import pytest
import torch

from src.kernels.linear import SMALL_M_MAX, linear, linear_tf32x3, tf32_split, uses_small_m_kernel, uses_tf32x3

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M", [1, 7, 16, 100, 128, 256])
@pytest.mark.parametrize("N,K", [(1600, 256), (256, 512), (1, 4), (3, 100), (257, 128), (48, 1024), (40, 2048)])
def test_matches_float64(M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M * 1000 + N + K)
    x = torch.randn(M, K, device="cuda", generator=g)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.05
    assert uses_small_m_kernel(x, w)
    y = linear(x, w)
    ref = (x.double() @ w.double().T).float()
    torch.testing.assert_close(y, ref, rtol=2e-5, atol=2e-5 * K ** 0.5)


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("N,K", [(4177, 1024), (1030, 2048), (9, 520), (5248, 1024)])
def test_small_batch_weight_stream_matches_float64(M, N, K):
    """1-8 batch rows at K 512-2048 take the weight-streaming path of
    m3_linear_f32 (weight-row counts not a multiple of the CTA's, K not a
    multiple of a warp's slice, and 8 rows x 2048 columns of staged batch)."""
    g = torch.Generator(device="cuda").manual_seed(17 * M + N + K)
    x = torch.randn(M, K, device="cuda", generator=g)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.05
    assert uses_small_m_kernel(x, w)
    torch.testing.assert_close(linear(x, w), (x.double() @ w.double().T).float(), rtol=2e-5, atol=2e-5 * K ** 0.5)


def test_strided_rows_and_views():
    x_big = torch.randn(64, 300, device="cuda")
    x = x_big[:, :256]  # row stride 300
    w_big = torch.randn(96, 260, device="cuda")
    w = w_big[:, :256]
    assert uses_small_m_kernel(x, w)
    torch.testing.assert_close(linear(x, w), (x.double() @ w.double().T).float(), rtol=2e-5, atol=4e-4)


def test_dispatch_outside_the_small_batch_regime():
    w = torch.randn(64, 128, device="cuda")
    big = torch.randn(SMALL_M_MAX + 1, 128, device="cuda")
    assert not uses_small_m_kernel(big, w)
    assert uses_tf32x3(big, w)
    torch.testing.assert_close(linear(big, w), (big.double() @ w.double().T).float(), rtol=1e-5, atol=1e-4)
    xb = torch.randn(8, 128, device="cuda").bfloat16()
    assert not uses_small_m_kernel(xb, w.bfloat16())
    torch.testing.assert_close(linear(xb, w.bfloat16()), xb @ w.bfloat16().T)
    # bf16 batches of up to SKINNY_ROUTE_M rows take the weight-streaming kernel
    from src.kernels import linear as lin
    assert 8 <= lin.SKINNY_ROUTE_M and uses_skinny_bf16(xb, w.bfloat16())
    assert torch.equal(linear(xb, w.bfloat16()), lin.linear_bf16_skinny(xb, w.bfloat16()))
    odd = torch.randn(8, 130, device="cuda")
    assert not uses_small_m_kernel(odd, torch.randn(4, 130, device="cuda"))


def test_empty_batch():
    out = linear(torch.zeros(0, 256, device="cuda"), torch.randn(32, 256, device="cuda"))
    assert out.shape == (0, 32)


# ---- bf16 projections on the tcgen05 GEMM (m3_linear_bf16) ----

from src.kernels.linear import TC_MAX_M, linear_bf16, uses_tc_bf16  # noqa: E402

TC_SHAPES = [  # M, N, K: the 24-layer stack's in_proj / out_proj, tails in every dimension, split-K
    (256, 9472, 2048), (256, 2048, 4096), (1, 128, 64), (7, 300, 136), (100, 4176, 512),
    (512, 512, 1024), (33, 1000, 1000), (300, 64, 72),
]


@pytest.mark.parametrize("M,N,K", TC_SHAPES)
def test_tc_bf16_matches_float64(M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + 7 * N + 13 * K)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    assert uses_tc_bf16(x, w)
    ref = x.double() @ w.double().T
    y32 = linear_bf16(x, w, torch.float32)
    # bf16 products are exact in fp32; the error is the fp32 accumulation's
    err = (y32.double() - ref).abs().max().item()
    assert err <= 2e-6 * K ** 0.5 * max(1.0, ref.abs().max().item()), err
    y = linear_bf16(x, w)
    assert y.dtype == torch.bfloat16 and y.shape == (M, N)
    assert torch.equal(y, y32.bfloat16()), "bf16 output is not the rounded fp32 result"


def test_tc_bf16_strided_rows():
    xb = torch.randn(64, 264, device="cuda").bfloat16()
    wb = (torch.randn(200, 272, device="cuda") * 0.05).bfloat16()
    x, w = xb[:, :256], wb[:, :256]
    assert uses_tc_bf16(x, w)
    ref = x.double() @ w.double().T
    torch.testing.assert_close(linear_bf16(x, w, torch.float32).double(), ref, rtol=0, atol=1e-4)


def test_tc_bf16_dispatch():
    w = torch.randn(64, 128, device="cuda").bfloat16()
    assert not uses_tc_bf16(torch.randn(TC_MAX_M + 1, 128, device="cuda").bfloat16(), w)
    assert not uses_tc_bf16(torch.randn(4, 128, device="cuda"), w.float())
    assert not uses_tc_bf16(torch.randn(4, 60, device="cuda").bfloat16(), torch.randn(8, 60, device="cuda").bfloat16())
    from src import _native as nat
    assert nat.device_error() == 0


# ---- fp32 projections of larger batches: split-precision tcgen05 GEMM ----

F32TC_SHAPES = [  # M, N, K: the d1024 layer's in_proj (R 4) / out_proj at batch 4096, tails, odd K, and the
    # mid-sized batches of that layer the tensor-core path takes below SMALL_M_MAX rows
    (4096, 5248, 1024), (4096, 1024, 2048), (257, 64, 32), (300, 1000, 100), (1000, 4480, 1024), (600, 257, 36),
    (513, 6272, 1024), (33, 4224, 1024), (64, 5248, 1024), (128, 1024, 2048), (200, 6272, 1024),
]


@pytest.mark.parametrize("M,N,K", F32TC_SHAPES)
def test_tf32x3_matches_float64(M, N, K):
    """Each product is taken as hi.hi + hi.lo + lo.hi of TF32 heads and
    remainders (the dropped lo.lo and the remainders' own TF32 rounding are
    ~2^-22 relative), accumulated in fp32: the error must stay at the size of
    an fp32 GEMM's, 2e-6 sqrt(K) of the outputs' scale (the bound the bf16
    GEMM's exact products are held to), and within a small factor of cuBLAS
    fp32 on the same inputs."""
    g = torch.Generator(device="cuda").manual_seed(M + 7 * N + 13 * K)
    x = torch.randn(M, K, device="cuda", generator=g)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.05
    assert uses_tf32x3(x, w)
    y = linear(x, w)
    assert y.dtype == torch.float32 and y.shape == (M, N)
    ref = x.double() @ w.double().T
    err = (y.double() - ref).abs().max().item()
    scale = max(1.0, ref.abs().max().item())
    assert err <= 2e-6 * K ** 0.5 * scale, err
    err_cublas = ((x @ w.T).double() - ref).abs().max().item()
    assert err <= 8.0 * err_cublas + 1e-6 * scale, (err, err_cublas)


def test_tf32x3_dispatch_for_mid_sized_batches():
    """Below SMALL_M_MAX rows the tensor-core path is taken only on large
    layers (K and N >= 1024) with enough work; small layers and the
    smallest batches keep the small-batch kernel."""
    from src.kernels.linear import TF32X3_MIN_ROWS, TF32X3_MIN_WORK
    w_in = torch.randn(5248, 1024, device="cuda") * 0.02
    w_out = torch.randn(1024, 2048, device="cuda") * 0.02
    assert uses_tf32x3(torch.randn(32, 1024, device="cuda"), w_in)
    assert not uses_tf32x3(torch.randn(TF32X3_MIN_ROWS - 1, 1024, device="cuda"), w_in)
    assert not uses_tf32x3(torch.randn(64, 2048, device="cuda"), w_out)  # 64 x 1024 < TF32X3_MIN_WORK
    assert 128 * 1024 >= TF32X3_MIN_WORK and uses_tf32x3(torch.randn(128, 2048, device="cuda"), w_out)
    assert not uses_tf32x3(torch.randn(200, 256, device="cuda"), torch.randn(1600, 256, device="cuda"))
    x = torch.randn(16, 1024, device="cuda")
    assert uses_small_m_kernel(x, w_in)
    torch.testing.assert_close(linear(x, w_in), (x.double() @ w_in.double().T).float(), rtol=2e-5, atol=2e-5 * 32)


def test_tf32_split_is_exact():
    x = torch.randn(300, 260, device="cuda") * 1e3
    hi, lo = tf32_split(x)
    assert torch.equal(hi + lo, x)
    assert torch.equal(hi.view(torch.int32) & 0x1FFF, torch.zeros_like(hi, dtype=torch.int32))
    assert (lo.abs() <= hi.abs() * 2.0 ** -10).all()


def test_tf32x3_strided_rows_and_weight_cache():
    xb = torch.randn(400, 136, device="cuda")
    wb = torch.randn(96, 140, device="cuda") * 0.05
    x, w = xb[:, :128], wb[:, :128]
    assert uses_tf32x3(x, w)
    ref = x.double() @ w.double().T
    torch.testing.assert_close(linear_tf32x3(x, w).double(), ref, rtol=0, atol=2e-5)
    w.mul_(2.0)  # an in-place change: the cached split must not be reused
    torch.testing.assert_close(linear_tf32x3(x, w).double(), 2.0 * ref, rtol=0, atol=4e-5)
    # a new weight in memory freed by an earlier one of the same shape
    ptr = w.data_ptr()
    del w, wb
    for _ in range(4):
        w2 = torch.randn(96, 140, device="cuda")[:, :128] * 0.05
        torch.testing.assert_close(linear_tf32x3(x, w2).double(), x.double() @ w2.double().T, rtol=0, atol=2e-5)
        if w2.data_ptr() == ptr:
            break
        del w2
    from src import _native as nat
    assert nat.device_error() == 0


# ---- bf16 projections of small batches: weight-streaming kernel ----

from src.kernels.linear import SKINNY_MAX_M, linear_bf16_skinny, uses_skinny_bf16  # noqa: E402

SKINNY_SHAPES = [  # M, N, K: the d2048 stack's in_proj / out_proj at 1..64 rows, tails in N and K
    (1, 9440, 2048), (8, 2048, 4096), (16, 9440, 2048), (17, 2048, 4096), (32, 9440, 2048), (32, 2048, 4096),
    (33, 1000, 1000), (48, 300, 136), (64, 9440, 2048), (64, 2048, 4096), (5, 7, 8), (64, 129, 4104),
    (3, 520, 24),
]


@pytest.mark.parametrize("M,N,K", SKINNY_SHAPES)
def test_skinny_bf16_matches_float64(M, N, K):
    """bf16 products are exact in fp32, so the error is the fp32
    accumulation's (the same bound as the tcgen05 GEMM's); the bf16 output
    is the rounded fp32 output."""
    g = torch.Generator(device="cuda").manual_seed(3 * M + 7 * N + 13 * K)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    assert uses_skinny_bf16(x, w)
    ref = x.double() @ w.double().T
    y32 = linear_bf16_skinny(x, w, torch.float32)
    err = (y32.double() - ref).abs().max().item()
    assert err <= 2e-6 * K ** 0.5 * max(1.0, ref.abs().max().item()), err
    y = linear_bf16_skinny(x, w)
    assert y.dtype == torch.bfloat16 and y.shape == (M, N)
    assert torch.equal(y, y32.bfloat16()), "bf16 output is not the rounded fp32 result"
    assert torch.equal(linear_bf16_skinny(x, w, torch.float32), y32), "not deterministic"


def test_skinny_bf16_strided_rows_and_output():
    xb = torch.randn(40, 264, device="cuda").bfloat16()
    wb = (torch.randn(200, 272, device="cuda") * 0.05).bfloat16()
    x, w = xb[:, :256], wb[:, :256]
    assert uses_skinny_bf16(x, w)
    ref = x.double() @ w.double().T
    torch.testing.assert_close(linear_bf16_skinny(x, w, torch.float32).double(), ref, rtol=0, atol=1e-4)
    # an output with a row stride wider than N (columns 200..207 untouched)
    from src import _native as nat
    out = torch.full((40, 208), 7.0, device="cuda")
    with nat.device_guard(x.device):
        st = nat.load().m3_linear_bf16_skinny(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(),
                                              208, 40, 200, 256, nat.M3_F32, nat.stream_handle(x.device))
    nat.check(st, "m3_linear_bf16_skinny")
    torch.testing.assert_close(out[:, :200].double(), ref, rtol=0, atol=1e-4)
    assert (out[:, 200:] == 7.0).all()


def test_skinny_bf16_rejects():
    from src import _native as nat
    lib = nat.load()
    x = torch.randn(SKINNY_MAX_M + 1, 128, device="cuda").bfloat16()
    w = torch.randn(64, 128, device="cuda").bfloat16()
    y = torch.empty(SKINNY_MAX_M + 1, 64, device="cuda")
    assert not uses_skinny_bf16(x, w)
    s = nat.stream_handle(x.device)
    assert lib.m3_linear_bf16_skinny(x.data_ptr(), 128, w.data_ptr(), 128, y.data_ptr(), 64, SKINNY_MAX_M + 1, 64,
                                     128, nat.M3_F32, s) == nat.M3_ERR_SHAPE
    assert lib.m3_linear_bf16_skinny(x.data_ptr(), 128, w.data_ptr(), 128, y.data_ptr(), 64, 4, 64, 124,
                                     nat.M3_F32, s) == nat.M3_ERR_ALIGN
    assert lib.m3_linear_bf16_skinny(x.data_ptr() + 2, 128, w.data_ptr(), 128, y.data_ptr(), 64, 4, 64, 120,
                                     nat.M3_F32, s) == nat.M3_ERR_ALIGN
    assert lib.m3_linear_bf16_skinny(x.data_ptr(), 128, w.data_ptr(), 128, y.data_ptr(), 64, 0, 64, 128,
                                     nat.M3_F32, s) == nat.M3_OK
    assert nat.device_error() == 0
