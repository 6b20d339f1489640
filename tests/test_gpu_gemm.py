"""tcgen05 projection GEMM (qkv_gemm_bf16, qkv_gemm_swiglu_bf16) against torch's f32 matmul of the
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


@pytest.mark.parametrize("m,n2,k", [(1, 256, 64), (7, 1024, 256), (33, 384, 512), (64, 12288, 2048),
                                    (32, 6144, 1024), (5, 6144, 1024), (17, 12288, 2048), (64, 1536, 4096),
                                    (300, 6144, 1024), (1000, 12288, 2048)])
def test_gemm_swiglu_epilogue(pkg, m, n2, k):
    """qkv_gemm_swiglu_bf16 (SwiGLU in the GEMM's epilogue, gate and up rows
    interleaved one by one), with and without a stream-K workspace, against
    torch: silu(g) * u of the f32 product of the same bf16 operands, g and u
    the even and odd rows.  Every output is written (NaN-filled beforehand)
    and within one bf16 rounding (2^-8 relative) of the reference, plus the
    GEMM's own 1e-4."""
    g_ = torch.Generator(device="cuda").manual_seed(m + n2 + k)
    x = torch.randn((m, k), device="cuda", generator=g_).to(torch.bfloat16)
    w = (0.05 * torch.randn((n2, k), device="cuda", generator=g_)).to(torch.bfloat16)
    gu = x.float() @ w.float().t()
    g, u = gu[:, 0::2], gu[:, 1::2]
    ref = g / (1.0 + torch.exp(-g)) * u
    # without and with a stream-K workspace (used where the output tiles would
    # leave SMs idle: the decode shapes here); the workspace call runs twice
    tiles = 2 * ((n2 + 127) // 128)
    ws = torch.empty(tiles * 4 * 128 * 64, device="cuda")
    flags = torch.zeros(tiles * 4, device="cuda", dtype=torch.int32)
    outs = []
    for use_ws in (False, True, True):
        act = torch.full((m, n2 // 2), float("nan"), device="cuda", dtype=torch.bfloat16)
        args = (ws.data_ptr(), flags.data_ptr(), ws.numel(), tiles) if use_ws else (None, None, 0, 0)
        assert pkg.lib.qkv_gemm_swiglu_bf16(x.data_ptr(), w.data_ptr(), act.data_ptr(), m, n2, k, *args, None) == 0
        torch.cuda.synchronize()
        got = act.float()
        assert torch.isfinite(got).all()
        err = ((got - ref).abs() / (ref.abs() + 1e-3 * ref.abs().max())).max().item()
        assert err < 2 ** -8 + 2e-4, (use_ws, err)
        outs.append(act)
    assert int(flags.abs().sum().item()) == 0          # counters left zero
    assert torch.equal(outs[1], outs[2])               # stream-K is deterministic


# ---- FP8 (e4m3) projections: qkv_quantize_rows_e4m3 + qkv_gemm_fp8 ----

def quantize_rows_torch(x_bf16):
    """The quantiser's definition: scale = amax / 448 per row (1 for a zero
    row), codes = RNE e4m3 of x * (1 / scale), saturated to +-448."""
    xf = x_bf16.float()
    amax = xf.abs().amax(dim=1, keepdim=True)
    # tensor / tensor: torch turns a division by a Python scalar into a
    # multiplication by its reciprocal, which is not the correctly rounded quotient
    scale = torch.where(amax > 0, amax / torch.full_like(amax, 448.0), torch.ones_like(amax))
    inv = torch.where(amax > 0, torch.ones_like(scale) / scale, torch.zeros_like(amax))
    codes = (xf * inv).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return codes, scale.squeeze(1)


def device_quantize(pkg, x_bf16):
    rows, k = x_bf16.shape
    codes = torch.empty((rows, k), dtype=torch.uint8, device="cuda")
    scales = torch.empty(rows, device="cuda")
    assert pkg.lib.qkv_quantize_rows_e4m3(x_bf16.data_ptr(), rows, k, codes.data_ptr(), scales.data_ptr(), None) == 0
    torch.cuda.synchronize()
    return codes, scales


def test_quantize_rows_e4m3_matches_definition(pkg):
    g = torch.Generator(device="cuda").manual_seed(17)
    x = torch.randn((300, 2048), device="cuda", generator=g)
    x[3] = 0.0                                # an all-zero row: scale 1, codes 0
    x[5, 7] = 1e4                             # one outlier row
    x[9] *= 1e-6                              # tiny values (e4m3 subnormals)
    xb = x.to(torch.bfloat16)
    codes, scales = device_quantize(pkg, xb)
    want_codes, want_scales = quantize_rows_torch(xb)
    assert torch.equal(scales, want_scales)
    assert torch.equal(codes, want_codes.view(torch.uint8))
    assert scales[3].item() == 1.0 and int(codes[3].abs().max().item()) == 0


FP8_SHAPES = [(1, 256, 128), (7, 1000, 256), (32, 4096, 1024), (32, 1024, 2048), (33, 384, 512), (64, 6144, 1024),
              (64, 2048, 6144), (129, 256, 128), (300, 4096, 1024), (512, 4096, 2048), (777, 2048, 6144),
              (1024, 12288, 2048)]


@pytest.mark.parametrize("m,n,k", FP8_SHAPES)
@pytest.mark.parametrize("accumulate", [0, 1])
def test_gemm_fp8_matches_dequantised_matmul(pkg, m, n, k, accumulate):
    """C (+)= (X x x_scale) . (W x w_scale)^T: e4m3 products are exact in f32,
    so against the f64 matmul of the dequantised operands the bar is f32
    accumulation, as for the bf16 GEMM (1e-4 relative)."""
    g = torch.Generator(device="cuda").manual_seed(m * 5 + n + k + accumulate)
    xq, xs = device_quantize(pkg, torch.randn((m, k), device="cuda", generator=g).to(torch.bfloat16))
    wq, ws = device_quantize(pkg, (0.05 * torch.randn((n, k), device="cuda", generator=g)).to(torch.bfloat16))
    base = torch.randn((m, n), device="cuda", generator=g) if accumulate else None
    c = base.clone() if accumulate else torch.full((m, n), float("nan"), device="cuda")
    rc = pkg.lib.qkv_gemm_fp8(xq.data_ptr(), xs.data_ptr(), wq.data_ptr(), ws.data_ptr(), c.data_ptr(), m, n, k,
                              accumulate, None)
    assert rc == 0
    torch.cuda.synchronize()
    xd = xq.view(torch.float8_e4m3fn).double() * xs.double()[:, None]
    wd = wq.view(torch.float8_e4m3fn).double() * ws.double()[:, None]
    ref = xd @ wd.t()
    if accumulate:
        ref = ref + base.double()
    err = ((c.double() - ref).abs().max() / ref.abs().max()).item()
    assert err < 1e-4, err


def test_gemm_fp8_rejects_k_not_multiple_of_128(pkg):
    t = torch.zeros(16, device="cuda")
    assert pkg.lib.qkv_gemm_fp8(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, 1, 64, 0,
                                None) != 0
