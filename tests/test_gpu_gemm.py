"""The tcgen05 GEMM engine against a torch fp32 reference GEMM of the same
bf16-rounded operands (all four operand majorness combinations, ragged
M / N / K tails, split-K accumulation)."""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def run_gemm(lib, M, N, K, a_k, b_k, engine, acc=False, seed=0, dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(dtype).cuda()
    B = torch.randn(N, K, generator=g).to(dtype).cuda()
    # storage layouts: K-major = row-major [rows, K]; MN-major = [K, rows]
    As = A.contiguous() if a_k else A.t().contiguous()
    Bs = B.contiguous() if b_k else B.t().contiguous()
    # pad the leading dimension to a multiple of 8 (16-byte rows)
    def pad(t):
        r, c = t.shape
        cp = (c + 7) // 8 * 8
        out = torch.zeros(r, cp, dtype=t.dtype, device=t.device)
        out[:, :c] = t
        return out
    As, Bs = pad(As), pad(Bs)
    Cm = torch.randn(M, N, generator=g).cuda() if acc else torch.zeros(M, N, device="cuda")
    ref = A.float() @ B.float().t() + (Cm if acc else 0)
    rc = lib.ptcg_gemm(M, N, K, C.c_void_p(As.data_ptr()), As.shape[1], int(a_k),
                       C.c_void_p(Bs.data_ptr()), Bs.shape[1], int(b_k),
                       1 if dtype == torch.bfloat16 else 0,
                       C.c_void_p(Cm.data_ptr()), N, int(acc), engine,
                       C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return rc, Cm, ref


@pytest.mark.parametrize("a_k,b_k", [(1, 1), (1, 0), (0, 0), (0, 1)])
@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (300, 144, 200), (1000, 768, 256),
                                   (129, 1024, 64), (4096, 300, 256), (514, 1536, 512),
                                   (514, 512, 2048), (514, 2048, 512), (1536, 512, 514),
                                   (1000, 256, 1024), (777, 200, 768)])
def test_tc_gemm_matches_fp32(pkg, a_k, b_k, M, N, K):
    """(the last two shapes: long-K GEMMs of at most 256 columns, the FFN1 /
    QKV dX form, with ragged M)"""
    import ptcg_b200.native as n
    lib = n.lib()
    if not lib.ptcg_tensor_cores():
        pytest.skip("no sm_100 device")
    rc, out, ref = run_gemm(lib, M, N, K, a_k, b_k, engine=1)
    assert lib.ptcg_device_error() == 0
    assert rc == 0, lib.ptcg_last_error()
    err = (out - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-3, err


@pytest.mark.parametrize("M,N,K", [(256, 768, 65536), (1024, 256, 20000)])
def test_tc_gemm_split_k_accumulate(pkg, M, N, K):
    """weight-gradient shape: both operands MN-major, long K, accumulate"""
    import ptcg_b200.native as n
    lib = n.lib()
    if not lib.ptcg_tensor_cores():
        pytest.skip("no sm_100 device")
    rc, out, ref = run_gemm(lib, M, N, K, 0, 0, engine=1, acc=True)
    assert lib.ptcg_device_error() == 0
    assert rc == 0, lib.ptcg_last_error()
    err = (out - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-3, err


@pytest.mark.parametrize("a_k,b_k", [(1, 1), (1, 0), (0, 0), (0, 1)])
@pytest.mark.parametrize("M,N,K", [(300, 144, 9000), (129, 1000, 3000), (640, 264, 4000),
                                   (1000, 256, 777)])
def test_tc_gemm_accumulate_row_pairs(pkg, a_k, b_k, M, N, K):
    """fp32-accumulate GEMMs run 256-row CTA tiles (two 128-row halves on one
    B stage): ragged M (a half past M, a tile half past M), every majorness,
    with and without the split over K"""
    import ptcg_b200.native as n
    lib = n.lib()
    if not lib.ptcg_tensor_cores():
        pytest.skip("no sm_100 device")
    rc, out, ref = run_gemm(lib, M, N, K, a_k, b_k, engine=1, acc=True, seed=M + K)
    assert lib.ptcg_device_error() == 0
    assert rc == 0, lib.ptcg_last_error()
    err = (out - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-3, err


def _tf32(x):
    """round-toward-zero to the 10-bit TF32 mantissa (what kind::tf32 reads)"""
    return (x.view(torch.int32) & ~0x1FFF).view(torch.float32)


@pytest.mark.parametrize("a_k,b_k", [(1, 1), (1, 0), (0, 0), (0, 1)])
@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (300, 144, 200), (4096, 256, 664),
                                   (1000, 960, 256), (256, 664, 40000)])
def test_tc_gemm_tf32(pkg, a_k, b_k, M, N, K):
    """fp32 operands on kind::tf32 (allowed through ptcg_gemm engine=3)"""
    import ptcg_b200.native as n
    lib = n.lib()
    if not lib.ptcg_tensor_cores():
        pytest.skip("no sm_100 device")
    rc, out, ref = run_gemm(lib, M, N, K, a_k, b_k, engine=3, dtype=torch.float32,
                            acc=(a_k == 0 and b_k == 0))
    assert lib.ptcg_device_error() == 0
    assert rc == 0, lib.ptcg_last_error()
    err = (out - ref).norm().item() / ref.norm().item()
    assert err < 2e-3, err


def test_fast_gelu_error_bound(pkg):
    """epilogue GELU / GELU' vs the exact erf form (torch, fp64)"""
    import ptcg_b200.native as n
    lib = n.lib()
    x = torch.linspace(-12, 12, 2_000_001, dtype=torch.float32, device="cuda")
    g = torch.empty_like(x); dg = torch.empty_like(x)
    assert lib.ptcg_eval_gelu(C.c_void_p(x.data_ptr()), C.c_void_p(g.data_ptr()),
                              C.c_void_p(dg.data_ptr()), x.numel(),
                              C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    xd = x.double()
    cdf = 0.5 * (1 + torch.erf(xd / 2 ** 0.5))
    pdf = torch.exp(-0.5 * xd * xd) / (2 * torch.pi) ** 0.5
    ref_g, ref_dg = xd * cdf, cdf + xd * pdf
    # degree-7 fit of the normal tail: |Phi error| <= 4e-6 (the activations
    # it feeds are stored in bf16, 2^-9 relative)
    eg = ((g.double() - ref_g).abs() / xd.abs().clamp(min=1)).max().item()
    edg = (dg.double() - ref_dg).abs().max().item()
    assert eg < 5e-6, eg
    assert edg < 6e-6, edg


@pytest.mark.parametrize("M,N,K", [(264192 // 16, 1024, 256), (1000, 1024, 256), (777, 1000, 256),
                                   (4099, 512, 128), (300, 96, 256), (20000, 768, 256)])
def test_tc_gemm_gelu_grad_epilogue(pkg, M, N, K):
    """the FFN2 dX form: bf16 out = (A B^T) * aux (the saved GELU'), fp32
    column sums of the product added into colsum (the FFN1 bias gradient);
    the last shape has 3 column tiles on a 148-CTA grid, so a CTA's tiles
    change columns"""
    import ptcg_b200.native as n
    lib = n.lib()
    if not lib.ptcg_tensor_cores():
        pytest.skip("no sm_100 device")
    g = torch.Generator(device="cpu").manual_seed(M + N + K)
    A = torch.randn(M, K, generator=g).bfloat16().cuda()
    B = torch.randn(N, K, generator=g).bfloat16().cuda()
    aux = torch.rand(M, N, generator=g).bfloat16().cuda()
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    colsum = torch.randn(N, generator=g).cuda()
    prod = (A.float() @ B.float().t()) * aux.float()
    ref_cs = colsum + prod.sum(0)
    rc = lib.ptcg_gemm_ex(M, N, K, C.c_void_p(A.data_ptr()), K, 1, C.c_void_p(B.data_ptr()), K, 1,
                          1, C.c_void_p(out.data_ptr()), N, 1, None, 2,
                          C.c_void_p(aux.data_ptr()), N, None, 0,
                          C.c_void_p(colsum.data_ptr()), 0, 1,
                          C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert lib.ptcg_device_error() == 0
    assert rc == 0, lib.ptcg_last_error()
    assert not out.float().isnan().any()
    err = (out.float() - prod).abs().max().item() / prod.abs().max().item()
    assert err < 1e-2, err      # bf16 output rounding
    cerr = (colsum - ref_cs).abs().max().item() / prod.abs().sum(0).max().item()
    assert cerr < 1e-4, cerr
