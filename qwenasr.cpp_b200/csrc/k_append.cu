// K1: fused K/V append.  One CTA per token row; 32 half-warp units, each
// holding 8 contiguous dims of one head (16 lanes x 8 = 128):
//   units  0..15  q heads  -> per-head RMSNorm -> NEOX RoPE -> q_out (f32) and/or
//                  q16_out (x scale, bf16/f16: the prefill kernel's Q operand)
//   units 16..23  k heads  -> per-head RMSNorm -> NEOX RoPE -> K page slot
//   units 24..31  v heads  -> raw                           -> V page slot
// Replaces text-decoder.cpp:375-433 (reshape, ggml_rms_norm * q/k_norm,
// ggml_rope_ext NEOX, permute + ggml_cpy into the cache view at n_past).
// The arithmetic is the scalar path's (:542-557 RMSNorm with a double mean
// square, :604-625 RoPE with a host-made double-angle cos/sin table), with
// every float op rounded on its own (__fmul_rn/__fadd_rn), so that given the
// same projections the stored K/V are bit-identical to the reference's cache.
// Each lane writes its 8 dims with one 16-byte store (bf16) / two (f32).
#include "kernels.h"

namespace qkv {

namespace {

template <typename TC> struct PageStore;
template <> struct PageStore<float> {
    static __device__ __forceinline__ void put(float *dst, const float (&v)[8], float) {
        reinterpret_cast<float4 *>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4 *>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
};
template <> struct PageStore<__nv_bfloat16> {
    static __device__ __forceinline__ void put(__nv_bfloat16 *dst, const float (&v)[8], float) {
        uint4 w;
        w.x = pack_bf16x2(v[0], v[1]);
        w.y = pack_bf16x2(v[2], v[3]);
        w.z = pack_bf16x2(v[4], v[5]);
        w.w = pack_bf16x2(v[6], v[7]);
        *reinterpret_cast<uint4 *>(dst) = w;
    }
};
template <> struct PageStore<uint8_t> {
    static __device__ __forceinline__ void put(uint8_t *dst, const float (&v)[8], float inv_scale) {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) lo |= static_cast<uint32_t>(f_to_e4m3(v[j] * inv_scale)) << (8 * j);
#pragma unroll
        for (int j = 0; j < 4; ++j) hi |= static_cast<uint32_t>(f_to_e4m3(v[4 + j] * inv_scale)) << (8 * j);
        *reinterpret_cast<uint2 *>(dst) = make_uint2(lo, hi);
    }
};

// V half of the e4m3-K / int8-V cache: excess-128 int8 bytes.
struct PageStoreI8 {
    static __device__ __forceinline__ void put(uint8_t *dst, const float (&v)[8], float inv_scale) {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) lo |= f_to_u8ex(v[j] * inv_scale) << (8 * j);
#pragma unroll
        for (int j = 0; j < 4; ++j) hi |= f_to_u8ex(v[4 + j] * inv_scale) << (8 * j);
        *reinterpret_cast<uint2 *>(dst) = make_uint2(lo, hi);
    }
};

// Per-head RMSNorm (double mean square, as text-decoder.cpp:542-557) and NEOX
// RoPE (:604-625) of the 8 dims a half-warp lane holds; lane l16 ^ 8 holds the
// rotation partners.  Must be called by all 32 lanes of the warp.
__device__ __forceinline__ void norm_rope8(float (&x)[8], const float *w8, const float2 *cs8, int l16, float eps) {
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += static_cast<double>(x[j]) * x[j];
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const double ms = ss / static_cast<double>(kHeadDim);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(ms), eps)));
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = __fmul_rn(__fmul_rn(x[j], scale), w8[j]);
    const bool lower = l16 < 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float other = __shfl_xor_sync(0xffffffffu, y[j], 8);
        const float2 t = cs8[j];
        if (lower) {  // row[i] = a*c - b*s   (a = own, b = partner)
            x[j] = __fsub_rn(__fmul_rn(y[j], t.x), __fmul_rn(other, t.y));
        } else {      // row[half+i] = b*c + a*s   (b = own, a = partner)
            x[j] = __fadd_rn(__fmul_rn(y[j], t.x), __fmul_rn(other, t.y));
        }
    }
}

template <typename TC>
__global__ void __launch_bounds__(512) kv_append_kernel(AppendParams p) {
    pdl_trigger();
    pdl_wait();   // everything below reads or writes memory of earlier kernels
    const int row = blockIdx.x;
    const int unit = threadIdx.x >> 4;      // 0..31
    const int l16 = threadIdx.x & 15;
    const int slot = p.slots[row];
    const int pos = p.positions[row];
    int page = -1;
    bool ok = slot >= 0 && slot < p.max_streams && pos >= 0 && pos < p.rope_len &&
              pos / kPageTokens < p.maxp;
    if (ok) {
        page = p.page_table[static_cast<size_t>(slot) * p.maxp + pos / kPageTokens];
        ok = page >= 0 && page < p.n_pages;
    }
    if (!ok) {  // block-uniform: nothing is written for this row
        if (threadIdx.x == 0) report_error(p.err, page < 0 ? kErrPosition : kErrPageIndex, kWhereAppend, row, pos);
        return;
    }

    int src_off;
    if (unit < kHq) src_off = unit * kHeadDim;
    else if (unit < kHq + kHkv) src_off = kQDim + (unit - kHq) * kHeadDim;
    else src_off = kQDim + kKvDim + (unit - kHq - kHkv) * kHeadDim;
    const float *src = p.qkv + static_cast<size_t>(row) * kQkvDim + src_off + l16 * 8;
    float x[8];
    {
        const float4 a = reinterpret_cast<const float4 *>(src)[0];
        const float4 b = reinterpret_cast<const float4 *>(src)[1];
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
    // The projection left one partial sum per K split: add them in slice order.
    for (int sl = 1; sl < p.qkv_slices; ++sl) {
        const float *ps = src + static_cast<size_t>(sl) * p.qkv_slice_stride;
        const float4 a = reinterpret_cast<const float4 *>(ps)[0];
        const float4 b = reinterpret_cast<const float4 *>(ps)[1];
        x[0] += a.x; x[1] += a.y; x[2] += a.z; x[3] += a.w;
        x[4] += b.x; x[5] += b.y; x[6] += b.z; x[7] += b.w;
    }

    // Warps 0-7 hold q units, 8-11 k units, 12-15 v units: the branch is warp-uniform.
    if (unit < kHq + kHkv) {
        // NEOX rotate-half: dim i (< 64) pairs with dim i + 64, held by lane l16 ^ 8.
        norm_rope8(x, (unit < kHq ? p.q_norm_w : p.k_norm_w) + l16 * 8,
                   p.rope + static_cast<size_t>(pos) * (kHeadDim / 2) + (l16 & 7) * 8, l16, p.eps);
    }

    if (unit < kHq) {
        const size_t off = static_cast<size_t>(row) * kQDim + unit * kHeadDim + l16 * 8;
        if (p.q16_out) {
            // Prefill rows for K3: q x scale rounded once to the MMA operand type.
            const float s = p.q16_scale;
            uint4 w;
            if (p.q16_f16) w = make_uint4(pack_h2(x[0] * s, x[1] * s), pack_h2(x[2] * s, x[3] * s),
                                          pack_h2(x[4] * s, x[5] * s), pack_h2(x[6] * s, x[7] * s));
            else w = make_uint4(pack_bf16x2(x[0] * s, x[1] * s), pack_bf16x2(x[2] * s, x[3] * s),
                                pack_bf16x2(x[4] * s, x[5] * s), pack_bf16x2(x[6] * s, x[7] * s));
            *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.q16_out) + off) = w;
        }
        if (p.q_out) {
            float *dst = p.q_out + off;
            reinterpret_cast<float4 *>(dst)[0] = make_float4(x[0], x[1], x[2], x[3]);
            reinterpret_cast<float4 *>(dst)[1] = make_float4(x[4], x[5], x[6], x[7]);
        }
        return;
    }
    const int kv = unit < kHq + kHkv ? 0 : 1;
    const int g = (unit - kHq) & (kHkv - 1);
    const int tok = pos & (kPageTokens - 1);
    float inv_scale = 1.0f;
    if constexpr (sizeof(TC) == 1) {
        // 8-bit caches: every stored (token, head) vector gets its own scale,
        // amax / qmax over its 128 elements (K after norm and RoPE, V raw), so
        // no stored token is ever re-quantised and no headroom is kept.
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(x[j]));
#pragma unroll
        for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float qmax = (kv == 1 && p.v_int8) ? kI8Max : kE4m3Max;
        const float scale = amax > 0.0f ? __fdiv_rn(amax, qmax) : 1.0f;
        inv_scale = amax > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
        if (l16 == 0)
            p.scales[((static_cast<size_t>(page) * 2 + kv) * kHkv + g) * kPageTokens + tok] = scale;
    }
    TC *pool = static_cast<TC *>(p.pool);
    TC *dst = pool + ((static_cast<size_t>(page) * 2 + kv) * kHkv + g) * (kPageTokens * kHeadDim) +
              tok * kHeadDim + l16 * 8;
    if constexpr (sizeof(TC) == 1) {
        if (kv == 1 && p.v_int8) {   // warp-uniform (warps 12..15 hold V)
            PageStoreI8::put(dst, x, inv_scale);
            return;
        }
    }
    PageStore<TC>::put(dst, x, inv_scale);
}

// Page gather: tokens [0, len) of one stream -> contiguous [len][Hkv*D] (K and V).
template <typename TC>
__global__ void page_gather_kernel(const TC *pool, const int *pages, int n_pages_row, int len, int n_pages,
                                   TC *k_out, TC *v_out, DevError *err) {
    const int tok = blockIdx.x;
    if (tok >= len) return;
    const int pi = tok / kPageTokens;
    const int page = pi < n_pages_row ? pages[pi] : -1;
    if (page < 0 || page >= n_pages) {
        if (threadIdx.x == 0) report_error(err, kErrPageIndex, kWhereGather, tok, page);
        return;
    }
    for (int e = threadIdx.x; e < kKvDim; e += blockDim.x) {
        const int g = e / kHeadDim, d = e % kHeadDim;
        const size_t k_off = ((static_cast<size_t>(page) * 2 + 0) * kHkv + g) * (kPageTokens * kHeadDim) +
                             (tok % kPageTokens) * kHeadDim + d;
        const size_t v_off = k_off + static_cast<size_t>(kPageHalfElems);
        k_out[static_cast<size_t>(tok) * kKvDim + e] = pool[k_off];
        v_out[static_cast<size_t>(tok) * kKvDim + e] = pool[v_off];
    }
}

// Copy whole pages (all layers are separate launches): dst[i] <- src[i].
__global__ void page_copy_kernel(uint4 *pool, const int *src, const int *dst, int n, size_t page_vec) {
    for (int i = blockIdx.y; i < n; i += gridDim.y) {
        const uint4 *s = pool + static_cast<size_t>(src[i]) * page_vec;
        uint4 *d = pool + static_cast<size_t>(dst[i]) * page_vec;
        for (size_t e = blockIdx.x * blockDim.x + threadIdx.x; e < page_vec; e += static_cast<size_t>(gridDim.x) * blockDim.x)
            d[e] = s[e];
    }
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Seeded N(0,1) fill of the given pages (Box-Muller on a counter hash).
// 8-bit caches: scale 8 / qmax per (page, K|V, head, token); v_int8 stores V as int8.
template <typename TC>
__global__ void page_fill_kernel(TC *pool, float *scales, const int *pages, int n, uint64_t seed, int v_int8) {
    const size_t per_page = static_cast<size_t>(2) * kPageHalfElems;
    for (int i = blockIdx.y; i < n; i += gridDim.y) {
        const int page = pages[i];
        TC *base = pool + static_cast<size_t>(page) * per_page;
        for (size_t e = blockIdx.x * blockDim.x + threadIdx.x; e < per_page; e += static_cast<size_t>(gridDim.x) * blockDim.x) {
            const uint64_t h = mix64(seed ^ mix64(static_cast<uint64_t>(page) * per_page + e + 0x1234567ull));
            const float u1 = (static_cast<float>(h >> 40) + 1.0f) * (1.0f / 16777217.0f);
            const float u2 = static_cast<float>((h >> 16) & 0xffffffu) * (1.0f / 16777216.0f);
            const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
            if constexpr (sizeof(TC) == 4) base[e] = z;
            else if constexpr (sizeof(TC) == 2) base[e] = __float2bfloat16_rn(z);
            else if (v_int8 && e >= static_cast<size_t>(kPageHalfElems)) base[e] = static_cast<uint8_t>(f_to_u8ex(z * (kI8Max / 8.0f)));
            else base[e] = f_to_e4m3(z * (kE4m3Max / 8.0f));
        }
        if constexpr (sizeof(TC) == 1) {
            if (blockIdx.x == 0) {
                for (int i = threadIdx.x; i < kPageScales; i += blockDim.x)
                    scales[static_cast<size_t>(page) * kPageScales + i] =
                        8.0f / (v_int8 && i >= kPageScales / 2 ? kI8Max : kE4m3Max);
            }
        }
    }
}

}  // namespace

cudaError_t launch_kv_append(const AppendParams &p, int kv_dtype, cudaStream_t st) {
    if (p.n <= 0) return cudaSuccess;
    switch (kv_dtype) {
        case kKvF32: return launch_pdl(kv_append_kernel<float>, dim3(p.n), dim3(512), 0, st, p);
        case kKvBF16: return launch_pdl(kv_append_kernel<__nv_bfloat16>, dim3(p.n), dim3(512), 0, st, p);
        case kKvFP8:
        case kKvE4I8: {
            AppendParams q = p;
            q.v_int8 = kv_dtype == kKvE4I8 ? 1 : 0;
            return launch_pdl(kv_append_kernel<uint8_t>, dim3(q.n), dim3(512), 0, st, q);
        }
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}


cudaError_t launch_page_gather(const void *pool, int kv_dtype, const int *pages, int n_pages_row, int len,
                               int n_pages, void *k_out, void *v_out, DevError *err, cudaStream_t st) {
    if (len <= 0) return cudaSuccess;
    switch (kv_dtype) {
        case kKvF32:
            page_gather_kernel<float><<<len, 256, 0, st>>>(static_cast<const float *>(pool), pages, n_pages_row, len,
                                                           n_pages, static_cast<float *>(k_out), static_cast<float *>(v_out), err);
            break;
        case kKvBF16:
            page_gather_kernel<__nv_bfloat16><<<len, 256, 0, st>>>(
                static_cast<const __nv_bfloat16 *>(pool), pages, n_pages_row, len, n_pages,
                static_cast<__nv_bfloat16 *>(k_out), static_cast<__nv_bfloat16 *>(v_out), err);
            break;
        case kKvFP8:
        case kKvE4I8:
            page_gather_kernel<uint8_t><<<len, 256, 0, st>>>(static_cast<const uint8_t *>(pool), pages, n_pages_row, len,
                                                             n_pages, static_cast<uint8_t *>(k_out), static_cast<uint8_t *>(v_out), err);
            break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_page_copy(void *pool_layer, size_t page_bytes, const int *src, const int *dst, int n,
                             cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const size_t vec = page_bytes / sizeof(uint4);
    dim3 grid(static_cast<unsigned>((vec + 255) / 256 < 64 ? (vec + 255) / 256 : 64), n < 1024 ? n : 1024);
    page_copy_kernel<<<grid, 256, 0, st>>>(static_cast<uint4 *>(pool_layer), src, dst, n, vec);
    return cudaGetLastError();
}

cudaError_t launch_page_fill(void *pool_layer, float *scales_layer, int kv_dtype, const int *pages, int n,
                             uint64_t seed, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    dim3 grid(32, n < 4096 ? n : 4096);
    switch (kv_dtype) {
        case kKvF32: page_fill_kernel<float><<<grid, 256, 0, st>>>(static_cast<float *>(pool_layer), nullptr, pages, n, seed, 0); break;
        case kKvBF16:
            page_fill_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<__nv_bfloat16 *>(pool_layer), nullptr, pages, n, seed, 0);
            break;
        case kKvFP8:
        case kKvE4I8:
            page_fill_kernel<uint8_t><<<grid, 256, 0, st>>>(static_cast<uint8_t *>(pool_layer), scales_layer, pages, n, seed,
                                                            kv_dtype == kKvE4I8 ? 1 : 0);
            break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace qkv
