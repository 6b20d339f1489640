// Causal prefill attention over the paged cache (CUDA cores).  Each query row
// (stream slot, position p) attends over keys [0, p] of its stream, which K1
// has already written into the pages.  Replaces the prompt half of
// text-decoder.cpp:322-334 (diag_mask_inf + soft_max_ext over P x P) and the
// scalar twin :739-791.  Block = one query row, warp g = kv head g serving
// q heads 2g, 2g+1; keys in groups of 32 (lane = key for QK, lane = 4 dims
// for PV), online softmax in the log2 domain.
#include "kernels.h"

namespace qkv {

namespace {

template <typename TC> __device__ __forceinline__ void load_row16(const TC *p, float (&o)[16]);
template <> __device__ __forceinline__ void load_row16<float>(const float *p, float (&o)[16]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float4 v = reinterpret_cast<const float4 *>(p)[k];
        o[4 * k] = v.x; o[4 * k + 1] = v.y; o[4 * k + 2] = v.z; o[4 * k + 3] = v.w;
    }
}
template <> __device__ __forceinline__ void load_row16<__nv_bfloat16>(const __nv_bfloat16 *p, float (&o)[16]) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint4 w = reinterpret_cast<const uint4 *>(p)[k];
        o[8 * k + 0] = bf16lo(w.x); o[8 * k + 1] = bf16hi(w.x); o[8 * k + 2] = bf16lo(w.y); o[8 * k + 3] = bf16hi(w.y);
        o[8 * k + 4] = bf16lo(w.z); o[8 * k + 5] = bf16hi(w.z); o[8 * k + 6] = bf16lo(w.w); o[8 * k + 7] = bf16hi(w.w);
    }
}
template <> __device__ __forceinline__ void load_row16<uint8_t>(const uint8_t *p, float (&o)[16]) {
    const uint4 w = *reinterpret_cast<const uint4 *>(p);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 a = e4m3x2_to_f2(static_cast<uint16_t>(ws[k] & 0xffffu));
        const float2 b = e4m3x2_to_f2(static_cast<uint16_t>(ws[k] >> 16));
        o[4 * k] = a.x; o[4 * k + 1] = a.y; o[4 * k + 2] = b.x; o[4 * k + 3] = b.y;
    }
}

template <typename TC> __device__ __forceinline__ float4 load_v4(const TC *p);
template <> __device__ __forceinline__ float4 load_v4<float>(const float *p) { return *reinterpret_cast<const float4 *>(p); }
template <> __device__ __forceinline__ float4 load_v4<__nv_bfloat16>(const __nv_bfloat16 *p) {
    const uint2 w = *reinterpret_cast<const uint2 *>(p);
    return make_float4(bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y));
}
template <> __device__ __forceinline__ float4 load_v4<uint8_t>(const uint8_t *p) {
    const uint32_t w = *reinterpret_cast<const uint32_t *>(p);
    const float2 a = e4m3x2_to_f2(static_cast<uint16_t>(w & 0xffffu));
    const float2 b = e4m3x2_to_f2(static_cast<uint16_t>(w >> 16));
    return make_float4(a.x, a.y, b.x, b.y);
}

// V of the e4m3-K / int8-V cache: four excess-128 int8 bytes.
__device__ __forceinline__ float4 load_v4_i8(const uint8_t *p) {
    const uint32_t w = *reinterpret_cast<const uint32_t *>(p);
    return make_float4(u8ex_to_f(w & 0xffu), u8ex_to_f((w >> 8) & 0xffu), u8ex_to_f((w >> 16) & 0xffu),
                       u8ex_to_f(w >> 24));
}

template <typename TOut> __device__ __forceinline__ void store_o4(TOut *p, float4 v);
template <> __device__ __forceinline__ void store_o4<float>(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
template <> __device__ __forceinline__ void store_o4<__nv_bfloat16>(__nv_bfloat16 *p, float4 v) {
    *reinterpret_cast<uint2 *>(p) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
}

template <typename TC, typename TOut, bool kVI8 = false>
__global__ void __launch_bounds__(256) prefill_attn_kernel(PrefillAttnParams p) {
    pdl_trigger();
    pdl_wait();   // everything below reads or writes memory of earlier kernels
    __shared__ __align__(16) float qs[kHkv][2][kHeadDim];
    const int row = blockIdx.x;
    const int g = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = p.slots[row], pos = p.positions[row];
    if (slot < 0 || slot >= p.max_streams || pos < 0 || pos / kPageTokens >= p.maxp) {
        if (threadIdx.x == 0) report_error(p.err, kErrRowBounds, kWherePrefillAttn, row, pos);
        return;
    }
    const float *qrow = p.q + static_cast<size_t>(row) * kQDim + 2 * g * kHeadDim;
    for (int e = lane; e < 2 * kHeadDim; e += 32) qs[g][e / kHeadDim][e % kHeadDim] = qrow[e] * p.scale_log2;
    __syncwarp();
    const TC *pool = static_cast<const TC *>(p.pool);
    const int *pt = p.page_table + static_cast<size_t>(slot) * p.maxp;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    float4 oa = make_float4(0.f, 0.f, 0.f, 0.f), ob = oa;
    for (int kb = 0; kb <= pos; kb += 32) {
        const int key = kb + lane;
        const bool valid = key <= pos;
        int page = 0;
        if (valid) {
            page = pt[key / kPageTokens];
            if (page < 0 || page >= p.n_pages) {
                report_error(p.err, kErrPageIndex, kWherePrefillAttn, row, page);
                page = 0;
            }
        }
        float sa = -INFINITY, sb = -INFINITY, sk = 1.f, sv = 1.f;
        if (valid) {
            const size_t kbase = ((static_cast<size_t>(page) * 2) * kHkv + g) * (kPageTokens * kHeadDim) +
                                 (key % kPageTokens) * kHeadDim;
            float da = 0.f, db = 0.f;
#pragma unroll
            for (int d0 = 0; d0 < kHeadDim; d0 += 16) {
                float kv[16];
                load_row16<TC>(pool + kbase + d0, kv);
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    da = fmaf(qs[g][0][d0 + e], kv[e], da);
                    db = fmaf(qs[g][1][d0 + e], kv[e], db);
                }
            }
            if constexpr (sizeof(TC) == 1) {   // the key's own (token, head) scales
                const size_t si = (static_cast<size_t>(page) * 2 * kHkv + g) * kPageTokens + key % kPageTokens;
                sk = p.scales[si];
                sv = p.scales[si + kHkv * kPageTokens];
            }
            sa = da * sk;
            sb = db * sk;
        }
        float ca = sa, cb = sb;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            ca = fmaxf(ca, __shfl_xor_sync(0xffffffffu, ca, o));
            cb = fmaxf(cb, __shfl_xor_sync(0xffffffffu, cb, o));
        }
        const float na = fmaxf(m_a, ca), nb = fmaxf(m_b, cb);
        const float pa = exp2f(sa - na), pb = exp2f(sb - nb);
        const float aa = exp2f(m_a - na), ab = exp2f(m_b - nb);
        float ta = pa, tb = pb;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            ta += __shfl_xor_sync(0xffffffffu, ta, o);
            tb += __shfl_xor_sync(0xffffffffu, tb, o);
        }
        l_a = l_a * aa + ta;
        l_b = l_b * ab + tb;
        m_a = na;
        m_b = nb;
        oa.x *= aa; oa.y *= aa; oa.z *= aa; oa.w *= aa;
        ob.x *= ab; ob.y *= ab; ob.z *= ab; ob.w *= ab;
        const float pva = pa * sv, pvb = pb * sv;
        const int nk = pos - kb + 1 < 32 ? pos - kb + 1 : 32;
        for (int jk = 0; jk < nk; ++jk) {
            const float wa = __shfl_sync(0xffffffffu, pva, jk);
            const float wb = __shfl_sync(0xffffffffu, pvb, jk);
            const int pg = __shfl_sync(0xffffffffu, page, jk);
            const int kk = kb + jk;
            const size_t vbase = ((static_cast<size_t>(pg) * 2 + 1) * kHkv + g) * (kPageTokens * kHeadDim) +
                                 (kk % kPageTokens) * kHeadDim + 4 * lane;
            float4 v;
            if constexpr (kVI8) v = load_v4_i8(reinterpret_cast<const uint8_t *>(pool) + vbase);
            else v = load_v4<TC>(pool + vbase);
            oa.x = fmaf(wa, v.x, oa.x); oa.y = fmaf(wa, v.y, oa.y); oa.z = fmaf(wa, v.z, oa.z); oa.w = fmaf(wa, v.w, oa.w);
            ob.x = fmaf(wb, v.x, ob.x); ob.y = fmaf(wb, v.y, ob.y); ob.z = fmaf(wb, v.z, ob.z); ob.w = fmaf(wb, v.w, ob.w);
        }
    }
    TOut *out = static_cast<TOut *>(p.out) + static_cast<size_t>(row) * kQDim + 2 * g * kHeadDim + 4 * lane;
    const float ia = 1.0f / l_a, ib = 1.0f / l_b;
    store_o4<TOut>(out, make_float4(oa.x * ia, oa.y * ia, oa.z * ia, oa.w * ia));
    store_o4<TOut>(out + kHeadDim, make_float4(ob.x * ib, ob.y * ib, ob.z * ib, ob.w * ib));
}

}  // namespace

cudaError_t launch_prefill_attn(const PrefillAttnParams &p, int kv_dtype, bool out_bf16, cudaStream_t st) {
    if (p.n <= 0) return cudaSuccess;
    switch (kv_dtype) {
        case kKvF32:
            if (out_bf16) return launch_pdl(prefill_attn_kernel<float, __nv_bfloat16>, dim3(p.n), dim3(256), 0, st, p);
            else return launch_pdl(prefill_attn_kernel<float, float>, dim3(p.n), dim3(256), 0, st, p);
            break;
        case kKvBF16:
            if (out_bf16) return launch_pdl(prefill_attn_kernel<__nv_bfloat16, __nv_bfloat16>, dim3(p.n), dim3(256), 0, st, p);
            else return launch_pdl(prefill_attn_kernel<__nv_bfloat16, float>, dim3(p.n), dim3(256), 0, st, p);
            break;
        case kKvFP8:
            if (out_bf16) return launch_pdl(prefill_attn_kernel<uint8_t, __nv_bfloat16>, dim3(p.n), dim3(256), 0, st, p);
            else return launch_pdl(prefill_attn_kernel<uint8_t, float>, dim3(p.n), dim3(256), 0, st, p);
            break;
        case kKvE4I8:
            if (out_bf16) return launch_pdl(prefill_attn_kernel<uint8_t, __nv_bfloat16, true>, dim3(p.n), dim3(256), 0, st, p);
            else return launch_pdl(prefill_attn_kernel<uint8_t, float, true>, dim3(p.n), dim3(256), 0, st, p);
            break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace qkv
