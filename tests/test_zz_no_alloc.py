"""The allocation-free decode-attention entry point (qkv_kv_attend_noalloc).

It serves callers that may not allocate device memory: the caller owns the KV
pool and page table (here: torch tensors standing in for a host framework's
own buffers) and the kernel's scratch comes from a fixed array in the library.
This test builds such a caller-owned pool from pages gathered out of a handle,
lays them out in a different page order, calls the entry point through the C
ABI twice in a row, and checks both outputs against qkv_kv_attend on the
handle's own pool.  It sits in its own file so that pytest collects it last."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

D, HQ, HKV, PT = 128, 16, 8, 16
QKV = (HQ + 2 * HKV) * D


def _i32(a):
    return torch.tensor(np.asarray(a, np.int32), device="cuda")


@pytest.mark.parametrize("kv", ["bf16", "f32", "fp8", "e4i8"])
def test_noalloc_attention_matches_handle_path(pkg, kv):
    kv_dtype = {"bf16": pkg.BF16, "f32": pkg.F32, "fp8": pkg.FP8, "e4i8": pkg.E4I8}[kv]
    elem = {"bf16": np.uint16, "f32": np.float32, "fp8": np.uint8, "e4i8": np.uint8}[kv]
    rng = np.random.default_rng(21)
    n_layers = 1
    qn = (1.0 + 0.1 * rng.standard_normal((n_layers, D))).astype(np.float32)
    kn = (1.0 + 0.1 * rng.standard_normal((n_layers, D))).astype(np.float32)
    cfg = dict(n_layers=n_layers, hidden=256, n_heads=HQ, n_kv_heads=HKV, head_dim=D, intermediate=512,
               vocab=1000, rope_theta=1.0e6, rms_norm_eps=1.0e-6)
    lens = [37, 300, 1200, 16, 1, 2049]
    rt = pkg.runtime_config(device=0, kv_dtype=kv_dtype, max_streams=len(lens), max_context=2100,
                            page_order_seed=4)
    with pkg.Decoder.kv_only(cfg, rt, qn, kn) as dec:
        streams = []
        for L in lens:
            s = dec.open()
            dec.extend(s, L)
            rows = torch.tensor(rng.standard_normal((L, QKV), dtype=np.float32), device="cuda")
            slots, pos = _i32([s] * L), _i32(np.arange(L))
            qtmp = torch.empty((L, HQ * D), device="cuda")
            dec.kv_append(0, L, slots.data_ptr(), pos.data_ptr(), rows.data_ptr(), qtmp.data_ptr())
            torch.cuda.synchronize()
            streams.append(s)
        dec.sync()
        q = torch.tensor(rng.standard_normal((len(lens), HQ * D), dtype=np.float32), device="cuda")
        d_slots, d_lens = _i32(streams), _i32(lens)
        want = torch.empty_like(q)
        dec.kv_attend(0, len(lens), d_slots.data_ptr(), d_lens.data_ptr(), q.data_ptr(), want.data_ptr())
        torch.cuda.synchronize()
        dec.sync()
        gathered = [dec.gather(0, s, kv_dtype) for s in streams]

    # The caller's own pool: same pages, reversed-permuted page ids.
    need = [(L + PT - 1) // PT for L in lens]
    n_pages = sum(need) + 3
    maxp = max(need)
    order = rng.permutation(n_pages)
    pool = np.zeros((n_pages, 2, HKV, PT, D), elem)
    scales = np.ones((n_pages, 2, HKV, PT), np.float32)
    table = np.full((len(lens), maxp), -1, np.int32)
    nxt = 0
    for i, (L, got) in enumerate(zip(lens, gathered)):
        k, v = got[0], got[1]
        for j in range(need[i]):
            page = int(order[nxt])
            nxt += 1
            table[i, j] = page
            t0, t1 = j * PT, min(L, (j + 1) * PT)
            pool[page, 0, :, : t1 - t0, :] = k[t0:t1].reshape(t1 - t0, HKV, D).transpose(1, 0, 2)
            pool[page, 1, :, : t1 - t0, :] = v[t0:t1].reshape(t1 - t0, HKV, D).transpose(1, 0, 2)
            if kv in ("fp8", "e4i8"):
                scales[page] = got[2][j]
    view = {"bf16": np.int16, "f32": np.float32, "fp8": np.uint8, "e4i8": np.uint8}[kv]
    d_pool = torch.tensor(pool.view(view), device="cuda")
    d_scales = torch.tensor(scales, device="cuda") if kv in ("fp8", "e4i8") else None
    d_table = torch.tensor(table, device="cuda")
    d_rows = _i32(np.arange(len(lens)))
    err = C.create_string_buffer(256)
    outs = []
    for _ in range(2):   # two calls in a row share (and reuse) the fixed scratch
        out = torch.full_like(q, float("nan"))
        rc = pkg.lib.qkv_kv_attend_noalloc(d_pool.data_ptr(), kv_dtype,
                                           d_scales.data_ptr() if d_scales is not None else None,
                                           d_table.data_ptr(), maxp, len(lens),
                                           n_pages, len(lens), d_rows.data_ptr(), d_lens.data_ptr(), q.data_ptr(),
                                           out.data_ptr(), None, err, 256)
        assert rc == 0, err.value.decode()
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
    ref = want.cpu().numpy()
    for got in outs:   # the same kernel on the same bytes: equal up to the split-row merge order
        rel = np.max(np.abs(got - ref)) / np.max(np.abs(ref))
        assert rel < 2e-5, rel


def test_noalloc_rejects_oversize_batch(pkg):
    err = C.create_string_buffer(256)
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = pkg.lib.qkv_kv_attend_noalloc(dummy.data_ptr(), pkg.BF16, None, dummy.data_ptr(), 1, 1, 1, 257,
                                       dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), None,
                                       err, 256)
    assert rc == 3 and b"256" in err.value
