"""The wide path's tcgen05 GEMM (cfb_wide_gemm) against a torch fp32 matmul of the same fp16
operands: every epilogue, ragged M (TMA zero fill past the edge) and N (zero rows of the packed
weights), split-K partials; and the weight packing (cfb_wide_pack) against its layout rule."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _pack(w):
    from chain_flow_b200 import _lib
    lib = _lib.load()
    buf = torch.empty(lib.cfb_wide_packed_bytes(w.shape[0], w.shape[1]), dtype=torch.uint8, device=w.device)
    _lib.check(lib.cfb_wide_pack(w.data_ptr(), w.stride(0), w.shape[0], w.shape[1], buf.data_ptr(),
                                 _lib.stream_ptr()), "cfb_wide_pack")
    return buf


def _gemm(a, w, bias, epi, splits=1, out_dtype=torch.float32, nsplit=1):
    from chain_flow_b200 import _lib
    lib = _lib.load()
    M, K = a.shape
    N = w.shape[0]
    wp = _pack(w)
    out = torch.zeros(nsplit, M, N, dtype=out_dtype, device=a.device).squeeze(0)
    err = torch.zeros(1, dtype=torch.int32, device=a.device)
    _lib.check(lib.cfb_wide_gemm(a.data_ptr(), a.stride(0), wp.data_ptr(), K,
                                 bias.data_ptr() if bias is not None else None, out.data_ptr(), N,
                                 M, N, K, epi, splits, err.data_ptr(), _lib.stream_ptr()), "cfb_wide_gemm")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


def _ref(a, w, bias):
    r = a.float() @ w.float().T
    return r + bias if bias is not None else r


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (1, 16, 64), (200, 384, 256), (300, 2560, 640),
                                   (37, 272, 2816), (768, 1024, 2560)])
def test_wide_gemm_f32_matches_torch(M, N, K):
    from chain_flow_b200 import _lib
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    a = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(N, device="cuda", generator=g)
    got = _gemm(a, w, bias, _lib.EPI_F32)
    want = _ref(a, w, bias)
    err = float((got - want).abs().max() / want.abs().max())
    assert err < 1e-4, err


def test_wide_gemm_half_gelu_and_strided_rows():
    from chain_flow_b200 import _lib
    g = torch.Generator(device="cuda").manual_seed(3)
    big = torch.randn(260, 512, device="cuda", generator=g).half()
    a = big[:, 64:320]                      # row stride 512, K = 256
    w = (torch.randn(96, 256, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(96, device="cuda", generator=g)
    want = _ref(a, w, bias)
    got16 = _gemm(a, w, bias, _lib.EPI_F16, out_dtype=torch.float16)
    assert float((got16.float() - want).abs().max()) < 2e-2
    gg = _gemm(a, w, bias, _lib.EPI_GELU16, out_dtype=torch.float16)
    assert float((gg.float() - torch.nn.functional.gelu(want)).abs().max()) < 2e-2


def test_wide_gemm_split_k_partials_sum_to_the_product():
    from chain_flow_b200 import _lib
    g = torch.Generator(device="cuda").manual_seed(4)
    M, N, K, S = 150, 256, 576, 3            # 9 k blocks -> 3 splits of 3
    a = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    parts = _gemm(a, w, None, _lib.EPI_PART, splits=S, nsplit=S)
    assert parts.shape == (S, M, N)
    for s in range(S):
        ks = slice(s * 192, (s + 1) * 192)
        want = a[:, ks].float() @ w[:, ks].float().T
        assert float((parts[s] - want).abs().max() / want.abs().max()) < 1e-4


def test_wide_pack_layout():
    """Block (n, j) of 256 rows x 64 columns at element (n * K/64 + j) * 16384; row r's 16-byte
    chunk c stored at chunk c ^ (r mod 8); rows past N zero."""
    N, K = 300, 192
    w = torch.arange(N * K, device="cuda", dtype=torch.float32).remainder(2039).half().view(N, K)
    got = _pack(w).view(torch.float16).view(2, K // 64, 256, 8, 8).cpu()
    wp = torch.zeros(512, K, dtype=torch.float16)
    wp[:N] = w.cpu()
    want = wp.view(2, 256, K // 64, 8, 8).permute(0, 2, 1, 3, 4)          # [nt, kb, r, chunk, 8]
    r = torch.arange(256).view(256, 1)
    c = torch.arange(8).view(1, 8)
    src = (c ^ (r % 8)).view(1, 1, 256, 8, 1).expand(2, K // 64, 256, 8, 8)
    assert torch.equal(got, torch.gather(want, 3, src))
