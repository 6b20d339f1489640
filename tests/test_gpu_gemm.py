"""tcgen05 projection GEMM (qkv_gemm_bf16) against torch's f32 matmul of the
same bf16 operands: decode shapes (split-K), prefill shapes (many token
tiles), ragged M/N edges, and accumulate mode."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SHAPES = [(1, 256, 64), (7, 1000, 256), (32, 4096, 1024), (32, 1024, 2048), (33, 384, 512), (64, 6144, 1024),
          (100, 1000, 256), (129, 256, 128), (300, 4096, 1024), (2000, 1024, 3072), (31, 151936, 1024)]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_matches_torch(pkg, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    x = torch.randn((m, k), device="cuda", generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn((n, k), device="cuda", generator=g)).to(torch.bfloat16)
    c = torch.full((m, n), float("nan"), device="cuda")
    rc = pkg.lib.qkv_gemm_bf16(x.data_ptr(), w.data_ptr(), c.data_ptr(), m, n, k, 0, None)
    assert rc == 0
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    err = (c - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-4, err


def test_gemm_accumulate(pkg):
    m, n, k = 20, 512, 1024
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn((m, k), device="cuda", generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn((n, k), device="cuda", generator=g)).to(torch.bfloat16)
    base = torch.randn((m, n), device="cuda", generator=g)
    c = base.clone()
    assert pkg.lib.qkv_gemm_bf16(x.data_ptr(), w.data_ptr(), c.data_ptr(), m, n, k, 1, None) == 0
    torch.cuda.synchronize()
    ref = base + x.float() @ w.float().t()
    assert ((c - ref).abs().max() / ref.abs().max()).item() < 1e-4
