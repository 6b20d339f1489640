"""tcgen05 projection GEMM (qkv_gemm_bf16) against torch's f32 matmul of the
same bf16 operands: decode shapes (split-K), prefill shapes (many token
tiles, several work units per persistent CTA so both TMEM accumulators
cycle), ragged M/N edges, accumulate mode (split red.add and unsplit
read-add-write), and bitwise repeatability of unsplit shapes."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SHAPES = [(1, 256, 64), (7, 1000, 256), (32, 4096, 1024), (32, 1024, 2048), (33, 384, 512), (64, 6144, 1024),
          (100, 1000, 256), (129, 256, 128), (300, 4096, 1024), (2000, 1024, 3072), (31, 151936, 1024),
          (512, 4096, 2048), (1024, 12288, 2048), (777, 2048, 6144), (1020, 151936, 2048)]


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


@pytest.mark.parametrize("m,n,k", [(20, 512, 1024), (512, 2048, 2048), (1000, 4096, 1024), (64, 2048, 6144)])
def test_gemm_accumulate(pkg, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn((m, k), device="cuda", generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn((n, k), device="cuda", generator=g)).to(torch.bfloat16)
    base = torch.randn((m, n), device="cuda", generator=g)
    c = base.clone()
    assert pkg.lib.qkv_gemm_bf16(x.data_ptr(), w.data_ptr(), c.data_ptr(), m, n, k, 1, None) == 0
    torch.cuda.synchronize()
    ref = base + x.float() @ w.float().t()
    assert ((c - ref).abs().max() / ref.abs().max()).item() < 1e-4


@pytest.mark.parametrize("m,n,k", [(512, 4096, 2048), (1024, 12288, 2048)])
def test_gemm_repeatable(pkg, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn((m, k), device="cuda", generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn((n, k), device="cuda", generator=g)).to(torch.bfloat16)
    outs = []
    for _ in range(2):
        c = torch.empty((m, n), device="cuda")
        assert pkg.lib.qkv_gemm_bf16(x.data_ptr(), w.data_ptr(), c.data_ptr(), m, n, k, 0, None) == 0
        torch.cuda.synchronize()
        outs.append(c)
    assert torch.equal(outs[0], outs[1])
