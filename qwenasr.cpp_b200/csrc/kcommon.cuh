// Device helpers shared by the sm_100a kernels: model constants, element
// conversions, the device error word, and thin inline-PTX wrappers for
// mbarriers and the bulk (non-tensor) async copy engine.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

namespace qkv {

// Qwen3 text-decoder attention geometry served by these kernels.
constexpr int kHeadDim = 128;   // head_dim
constexpr int kHq = 16;         // query heads
constexpr int kHkv = 8;         // kv heads (GQA 2:1)
constexpr int kPageTokens = 16; // tokens per KV page
constexpr int kQkvDim = (kHq + 2 * kHkv) * kHeadDim;   // 4096
constexpr int kQDim = kHq * kHeadDim;                   // 2048
constexpr int kKvDim = kHkv * kHeadDim;                 // 1024
// Elements of one (page, K|V) block: [kHkv][kPageTokens][kHeadDim].
constexpr int kPageHalfElems = kHkv * kPageTokens * kHeadDim;   // 16384
// 8-bit caches: one f32 scale per (page, K|V, kv head, token) = 256 per page.
constexpr int kPageScales = 2 * kHkv * kPageTokens;

// Device error word: first error wins.  The host reads it after a sync.
struct DevError {
    int code;    // 0 = none
    int where;   // kernel id
    int a, b;    // detail (index, value)
};
enum DevErrCode { kErrPageIndex = 1, kErrWaitTimeout = 2, kErrPosition = 3, kErrRowBounds = 4 };
enum DevErrWhere { kWhereAppend = 1, kWhereAttend = 2, kWherePrefillAttn = 3, kWhereGather = 4,
                   kWhereEmbed = 5, kWhereGemm = 6, kWhereProbe = 7 };

__device__ __forceinline__ void report_error(DevError *e, int code, int where, int a, int b) {
    if (e && atomicCAS(&e->code, 0, code) == 0) {
        e->where = where;
        e->a = a;
        e->b = b;
    }
}

// ---- element conversions ----
template <typename T> struct Elem;
template <> struct Elem<float> {
    static __device__ __forceinline__ float load(const float *p) { return *p; }
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

// Two e4m3 bytes (low byte first) -> two floats.
__device__ __forceinline__ float2 e4m3x2_to_f2(uint16_t v) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v), __NV_E4M3);
    const __half2 hh = *reinterpret_cast<const __half2 *>(&h);
    return __half22float2(hh);
}
// Two e4m3 bytes (low byte first) -> f16x2 bits (low half = low byte); exact.
__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint16_t v) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v), __NV_E4M3);
    uint32_t bits;
    memcpy(&bits, &h, sizeof(bits));
    return bits;
}
// Four e4m3 bytes -> two f16x2 words (bytes 0,1 -> lo2; bytes 2,3 -> hi2); exact.
// The word is split into its 16-bit halves inside PTX (no shift/mask ops).
__device__ __forceinline__ void e4m3x4_to_h2x2(uint32_t w, uint32_t &lo2, uint32_t &hi2) {
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, l;\n\tcvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
        : "=r"(lo2), "=r"(hi2) : "r"(w));
}
// acc += lo(a) * lo(b) + hi(a) * hi(b): f16 operands, products exact in f32,
// f32 accumulation (PTX fma.rn.f32.f16, sm_100).
__device__ __forceinline__ void dot2_f16_f32(float &acc, uint32_t a, uint32_t b) {
    asm("{\n\t.reg .f16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.f16 %0, al, bl, %0;\n\tfma.rn.f32.f16 %0, ah, bh, %0;\n\t}"
        : "+f"(acc) : "r"(a), "r"(b));
}
// acc0 += lo(v) * p, acc1 += hi(v) * p with p = half H (0 low, 1 high) of pw.
template <int H> __device__ __forceinline__ void axpy2_f16_f32(float &acc0, float &acc1, uint32_t v, uint32_t pw) {
    if constexpr (H == 0) {
        asm("{\n\t.reg .f16 vl, vh, pl, ph;\n\tmov.b32 {vl, vh}, %2;\n\tmov.b32 {pl, ph}, %3;\n\t"
            "fma.rn.f32.f16 %0, vl, pl, %0;\n\tfma.rn.f32.f16 %1, vh, pl, %1;\n\t}"
            : "+f"(acc0), "+f"(acc1) : "r"(v), "r"(pw));
    } else {
        asm("{\n\t.reg .f16 vl, vh, pl, ph;\n\tmov.b32 {vl, vh}, %2;\n\tmov.b32 {pl, ph}, %3;\n\t"
            "fma.rn.f32.f16 %0, vl, ph, %0;\n\tfma.rn.f32.f16 %1, vh, ph, %1;\n\t}"
            : "+f"(acc0), "+f"(acc1) : "r"(v), "r"(pw));
    }
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 v = __floats2half2_rn(lo, hi);
    uint32_t bits;
    memcpy(&bits, &v, sizeof(bits));
    return bits;
}
__device__ __forceinline__ uint8_t f_to_e4m3(float v) {
    return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}
constexpr float kE4m3Max = 448.0f;

// ---- int8 V of the e4m3-K / int8-V cache ----
// A V element is one excess-128 byte u = q + 128 with q = round(v / scale)
// clamped to [-127, 127], so u is 1..255.
constexpr float kI8Max = 127.0f;
__device__ __forceinline__ uint32_t f_to_u8ex(float v) {
    int q = __float2int_rn(v);
    q = q < -127 ? -127 : (q > 127 ? 127 : q);
    return static_cast<uint32_t>(q + 128);
}
__device__ __forceinline__ float u8ex_to_f(uint32_t u) { return static_cast<float>(static_cast<int>(u) - 128); }
// Four excess-128 bytes -> two f16x2 words holding q exactly (bytes 0,1 ->
// lo2; 2,3 -> hi2): 0x6400 | u is the f16 number 1024 + u, and subtracting
// 1152 (f16 bits 0x6480) leaves u - 128 = q.
__device__ __forceinline__ void u8x4_to_h2x2(uint32_t w, uint32_t &lo2, uint32_t &hi2) {
    const uint32_t a = __byte_perm(w, 0x64646464u, 0x4140);   // u0, 0x64, u1, 0x64
    const uint32_t b = __byte_perm(w, 0x64646464u, 0x4342);   // u2, 0x64, u3, 0x64
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(lo2) : "r"(a), "r"(0x64806480u));
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(hi2) : "r"(b), "r"(0x64806480u));
}

// ---- shared-memory address + mbarrier + bulk copy (inline PTX) ----
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase of `parity` to complete, for at most `limit` SM cycles.
// Returns false when the limit ran out (the caller records an error and stops).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) return false;
    }
    return true;
}

// Global -> shared bulk copy completing on `bar` (bytes: multiple of 16,
// both addresses 16-byte aligned).  No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// L2 policy: KV pages are streamed once per step -> evict first.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Programmatic dependent launch.  A kernel launched with it may start while the
// previous kernel of the stream is still running: pdl_trigger lets the next
// kernel start early, and pdl_wait blocks until the previous kernel has
// completed and its memory is visible (it returns at once for a normal launch).
// Every kernel below calls pdl_wait before its first access to memory that an
// earlier kernel of the stream wrote or reads.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Cycle budget for any single wait before it is treated as a hang (~2 s at 1.9 GHz).
constexpr long long kWaitLimitCycles = 4000000000ll;

}  // namespace qkv
