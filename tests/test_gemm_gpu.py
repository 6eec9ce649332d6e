"""GPU: the tcgen05 W4A16 / dense GEMM against torch fp32 references.

Two checks per case: (1) against the exact fp32 dequantisation
w = (nibble - 8) * scale (the reference test's semantics,
tests/unit/test_int4_dequant.py:18-53) with the max error relative to the
largest output <= 1e-2; (2) against an fp32 GEMM over the weights rounded as the reference rounds
them (fp32 dequantisation cast once to bf16, int4_dequant_triton.py:66),
max relative error <= 5e-3 (bf16 output rounding; catches any indexing error
the looser bound might hide); (3) the kernel's dequantised weights equal
those reference-rounded weights bit for bit (identity activations)."""
import pytest
import torch

from cudaforge_b200.gemm import dense_gemm, dequant_reference, pack_int4_reference, repack_int4, w4a16_gemm

pytestmark = pytest.mark.gpu


def _w4(K, N, seed, scale=0.002):
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(0, 16, (K, N), generator=g)
    s = (torch.randn(K // 128, N, generator=g).abs() * scale).to(torch.float16)
    return pack_int4_reference(q), s, q


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-20)).item()


@pytest.mark.parametrize("M,N,K", [(16, 128, 128), (64, 256, 512), (16, 256, 128), (64, 128, 512),
                                   (384, 6144, 4096), (100, 384, 1024), (640, 256, 1024), (1000, 128, 256),
                                   (1, 128, 128), (24, 4096, 14336)])
@pytest.mark.parametrize("split", [0, 1])
def test_w4a16_vs_fp32(M, N, K, split):
    wq, s, q = _w4(K, N, M + N + K)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    wd = dequant_reference(wq, s)
    ref = x.float() @ wd
    wk = repack_int4(wq.cuda())
    y = w4a16_gemm(x.cuda(), wk, s.cuda(), split_k=split)
    torch.cuda.synchronize()
    assert _rel(y.cpu(), ref) < 1e-2
    # the reference's weight rounding (int4_dequant_triton.py:66): the exact fp32 product
    # (q - 8) * scale cast once to the activation type
    w_bf = dequant_reference(wq, s).to(torch.bfloat16).float()
    ref2 = x.float() @ w_bf
    assert _rel(y.cpu(), ref2) < 5e-3  # bf16 output rounding is 2^-9 relative


def test_w4a16_weight_rounding_matches_reference():
    """x = identity rows picks single weight rows out of the GEMM: y[m, n] is then
    exactly the kernel's dequantised w[k=m, n] (one non-zero product, fp32
    accumulation, bf16 output of a bf16 value), which must equal the reference's
    bf16((q - 8) * float(scale)) bit for bit -- scales cover normal and subnormal
    fp16 values."""
    K, N = 256, 256
    g = torch.Generator().manual_seed(11)
    q = torch.randint(0, 16, (K, N), generator=g)
    s = (torch.randn(K // 128, N, generator=g).abs() * 0.002)
    s[:, :32] = torch.rand(K // 128, 32, generator=g) * 6e-5   # subnormal fp16 scales
    s[:, 32:64] = torch.rand(K // 128, 32, generator=g) * 8.0  # large scales
    s = s.to(torch.float16)
    wq = pack_int4_reference(q)
    x = torch.eye(K, dtype=torch.bfloat16)
    y = w4a16_gemm(x.cuda(), repack_int4(wq.cuda()), s.cuda())
    torch.cuda.synchronize()
    ref = dequant_reference(wq, s).to(torch.bfloat16)
    assert torch.equal(y.cpu(), ref)


def test_w4a16_residual_and_strided_out():
    M, N, K = 48, 512, 768
    wq, s, q = _w4(K, N, 3)
    x = torch.randn(M, K).to(torch.bfloat16)
    r = torch.randn(M, N).to(torch.bfloat16)
    out = torch.zeros(M, N + 64, dtype=torch.bfloat16).cuda()
    for split in (1, 3):
        y = w4a16_gemm(x.cuda(), repack_int4(wq.cuda()), s.cuda(), residual=r.cuda(), out=out[:, :N], split_k=split)
        torch.cuda.synchronize()
        ref = x.float() @ dequant_reference(wq, s) + r.float()
        assert _rel(y.cpu(), ref) < 1e-2
        assert (out[:, N:] == 0).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(32, 512, 512), (160, 1408, 512), (40, 32000, 512), (8, 128, 1408)])
def test_dense_vs_fp32(dtype, M, N, K):
    if N % 128:
        pytest.skip("N must be a multiple of 128")
    g = torch.Generator().manual_seed(M * N)
    x = torch.randn(M, K, generator=g).to(dtype)
    w = (torch.randn(N, K, generator=g) * 0.02).to(dtype)
    y = dense_gemm(x.cuda(), w.cuda())
    torch.cuda.synchronize()
    ref = x.float() @ w.float().T
    assert _rel(y.cpu(), ref) < 5e-3


def test_repack_roundtrip_values():
    wq, s, q = _w4(256, 128, 9)
    wk = repack_int4(wq.cuda()).cpu()
    w = wk.to(torch.int64) & 0xFFFFFFFF
    ks = [0, 2, 4, 6, 1, 3, 5, 7]
    orig = wq.to(torch.int64) & 0xFFFFFFFF
    for pos in range(8):
        assert torch.equal((w >> (4 * pos)) & 0xF, (orig >> (4 * ks[pos])) & 0xF)



@pytest.mark.parametrize("M,N,K,split", [(384, 4096, 14336, 0), (384, 6144, 4096, 0), (200, 1280, 2048, 5),
                                         (16, 128, 4096, 7)])
def test_split_k_deterministic(M, N, K, split):
    """Split-K partials are summed in a fixed order by the reduction kernel, so
    repeated calls are bit-identical (and match the fp32 reference)."""
    wq, s, q = _w4(K, N, 7)
    x = (torch.randn(M, K, generator=torch.Generator().manual_seed(2)) * 0.5).to(torch.bfloat16).cuda()
    wk, sc = repack_int4(wq.cuda()), s.cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ys = [w4a16_gemm(x, wk, sc, split_k=split, status=status).clone() for _ in range(3)]
    torch.cuda.synchronize()
    assert status.item() == 0
    assert all(torch.equal(ys[0], y) for y in ys[1:])
    ref = x.float().cpu() @ dequant_reference(wq, s)
    assert _rel(ys[0].cpu(), ref) < 1e-2
