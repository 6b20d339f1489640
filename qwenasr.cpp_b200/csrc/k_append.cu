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

#include "kappend.cuh"

namespace qkv {

namespace {

template <typename TC>
__global__ void __launch_bounds__(512) kv_append_kernel(AppendParams p) {
    pdl_trigger();
    pdl_wait();   // everything below reads or writes memory of earlier kernels
    append_row_unit<TC>(p, blockIdx.x, threadIdx.x >> 4, threadIdx.x & 15);
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
