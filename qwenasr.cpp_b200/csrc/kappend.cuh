// The arithmetic of K1, the K/V append (one token row: QK-RMSNorm, RoPE,
// page store), shared by kv_append_kernel and the append-ahead of K2
// (decode_attn_kernel with AttendParams::next), so both write the same
// bytes.  Follows text-decoder.cpp:542-557 (RMSNorm with a double mean
// square) and :604-625 (NEOX RoPE with the host-made cos/sin table), every
// float op rounded on its own (__fmul_rn / __fadd_rn), so that given the same
// projections the stored K/V are bit-identical to the reference's cache.
#pragma once

#include "kernels.h"

namespace qkv {

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

// 8 consecutive floats of a projection row that may be split into partial-sum
// slices (the K-split GEMM's slice mode): slice 0, then the others added in
// slice order.
__device__ __forceinline__ void load_row8(const float *src, int slices, size_t slice_stride, float (&x)[8]) {
    {
        const float4 a = reinterpret_cast<const float4 *>(src)[0];
        const float4 b = reinterpret_cast<const float4 *>(src)[1];
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
    for (int sl = 1; sl < slices; ++sl) {
        const float *ps = src + static_cast<size_t>(sl) * slice_stride;
        const float4 a = reinterpret_cast<const float4 *>(ps)[0];
        const float4 b = reinterpret_cast<const float4 *>(ps)[1];
        x[0] += a.x; x[1] += a.y; x[2] += a.z; x[3] += a.w;
        x[4] += b.x; x[5] += b.y; x[6] += b.z; x[7] += b.w;
    }
}

// Per-head RMSNorm and NEOX RoPE of the 8 dims a half-warp lane holds
// (lane l16 of 16 holds dims [8 l16, 8 l16 + 8)); lane l16 ^ 8 holds the
// rotation partners (dim i < 64 pairs with dim i + 64).  cs8 = the (cos, sin)
// of the lane's 8 pair indices.  Must be called by all 32 lanes of the warp.
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

// One half-warp unit of a token's append: the 8 raw projection dims x that
// lane l16 holds of K (kv = 0: QK-RMSNorm with k_norm_w and RoPE at pos
// first) or V (kv = 1: stored raw) of kv head g, stored into token slot
// pos % 16 of `page`.  8-bit caches: every stored (token, head) vector gets
// its own scale, amax / qmax over its 128 elements (qmax 448 for e4m3, 127
// for int8 V), written to scales, so no stored token is ever re-quantised and
// no headroom is kept.  kv must be the same for all 32 lanes of the warp
// (the RoPE and amax exchanges run over each half-warp).
template <typename TC>
__device__ __forceinline__ void append_kv_unit(float (&x)[8], int kv, int g, int l16, int pos, int page, void *pool_v,
                                               float *scales, const float *k_norm_w, const float2 *rope, float eps,
                                               int v_int8) {
    if (kv == 0) norm_rope8(x, k_norm_w + l16 * 8, rope + static_cast<size_t>(pos) * (kHeadDim / 2) + (l16 & 7) * 8,
                            l16, eps);
    const int tok = pos & (kPageTokens - 1);
    float inv_scale = 1.0f;
    if constexpr (sizeof(TC) == 1) {
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(x[j]));
#pragma unroll
        for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float qmax = (kv == 1 && v_int8) ? kI8Max : kE4m3Max;
        const float scale = amax > 0.0f ? __fdiv_rn(amax, qmax) : 1.0f;
        inv_scale = amax > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
        if (l16 == 0) scales[((static_cast<size_t>(page) * 2 + kv) * kHkv + g) * kPageTokens + tok] = scale;
    }
    TC *dst = static_cast<TC *>(pool_v) + ((static_cast<size_t>(page) * 2 + kv) * kHkv + g) * (kPageTokens * kHeadDim) +
              tok * kHeadDim + l16 * 8;
    if constexpr (sizeof(TC) == 1) {
        if (kv == 1 && v_int8) {
            PageStoreI8::put(dst, x, inv_scale);
            return;
        }
    }
    PageStore<TC>::put(dst, x, inv_scale);
}

// K1's work for one half-warp unit of one row (32 units per row, 16 lanes x
// 8 dims each): units 0..15 q heads -> per-head RMSNorm -> NEOX RoPE ->
// q_out (f32) and/or q16_out (x q16_scale, bf16 or f16: K3's Q operand);
// units 16..23 K heads and 24..31 V heads -> append_kv_unit.  Units 2w and
// 2w + 1 must be called together by the 32 lanes of a warp (the pair is
// always of one kind).  A row whose slot, position or page is out of range
// writes nothing and is reported once (by unit 0).
template <typename TC>
__device__ __forceinline__ void append_row_unit(const AppendParams &p, int row, int unit, int l16) {
    const int slot = p.slots[row];
    const int pos = p.positions[row];
    int page = -1;
    bool ok = slot >= 0 && slot < p.max_streams && pos >= 0 && pos < p.rope_len && pos / kPageTokens < p.maxp;
    if (ok) {
        page = p.page_table[static_cast<size_t>(slot) * p.maxp + pos / kPageTokens];
        ok = page >= 0 && page < p.n_pages;
    }
    if (!ok) {   // uniform over the row: nothing is written for it
        if (unit == 0 && l16 == 0) report_error(p.err, page < 0 ? kErrPosition : kErrPageIndex, kWhereAppend, row, pos);
        return;
    }
    int src_off;
    if (unit < kHq) src_off = unit * kHeadDim;
    else if (unit < kHq + kHkv) src_off = kQDim + (unit - kHq) * kHeadDim;
    else src_off = kQDim + kKvDim + (unit - kHq - kHkv) * kHeadDim;
    float x[8];
    // The projection may have left one partial sum per K split: added in slice order.
    load_row8(p.qkv + static_cast<size_t>(row) * kQkvDim + src_off + l16 * 8, p.qkv_slices, p.qkv_slice_stride, x);
    if (unit < kHq) {
        norm_rope8(x, p.q_norm_w + l16 * 8, p.rope + static_cast<size_t>(pos) * (kHeadDim / 2) + (l16 & 7) * 8, l16,
                   p.eps);
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
    append_kv_unit<TC>(x, unit < kHq + kHkv ? 0 : 1, (unit - kHq) & (kHkv - 1), l16, pos, page, p.pool, p.scales,
                       p.k_norm_w, p.rope, p.eps, p.v_int8);
}

}  // namespace qkv
