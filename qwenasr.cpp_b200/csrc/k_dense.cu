// Dense per-token kernels of the decoder block around the KV-cache path:
// RMSNorm (text-decoder.cpp:542-557), embedding-row gather (:2297 / :2167),
// projections (:559-598, W[out][in] row-major), SwiGLU (:600, :794-797) and
// the first-maximum argmax of the greedy loop (:2266-2274).
#include "kernels.h"

#include <algorithm>

#include <cuda_fp16.h>

namespace qkv {

namespace {

template <typename T> __device__ __forceinline__ void put(T *p, float v);
template <> __device__ __forceinline__ void put<float>(float *p, float v) { *p = v; }
template <> __device__ __forceinline__ void put<__nv_bfloat16>(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

// Four outputs from a float4 (one 16-byte f32 or 8-byte bf16 store).
template <typename T> __device__ __forceinline__ void put4(T *p, float4 v);
template <> __device__ __forceinline__ void put4<float>(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
template <> __device__ __forceinline__ void put4<__nv_bfloat16>(__nv_bfloat16 *p, float4 v) {
    *reinterpret_cast<uint2 *>(p) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
}

// RMSNorm of one row per CTA (mean square accumulated in double, as the
// scalar path does).  Rows whose width is a multiple of 4 and at most
// 256 x 4 x kVec, with 16-byte aligned x and w, stay in registers between the
// two passes (one read of x, 16-byte loads); others take the element loop.
template <typename TOut>
__global__ void __launch_bounds__(256) rmsnorm_kernel(float *x, const int *rows, int hidden, const float *w,
                                                      float eps, TOut *out, ResidualFold fold) {
    constexpr int kVec = 4;
    pdl_trigger();
    pdl_wait();   // everything below reads or writes memory of earlier kernels
    const int r = blockIdx.x;
    const size_t xrow = static_cast<size_t>(rows ? rows[r] : r) * hidden;
    float *xr = x + xrow;
    TOut *o = out + static_cast<size_t>(r) * hidden;
    const bool vec = (hidden & 3) == 0 && hidden <= 256 * 4 * kVec &&
                     ((reinterpret_cast<uintptr_t>(xr) | reinterpret_cast<uintptr_t>(w)) & 15u) == 0 &&
                     (reinterpret_cast<uintptr_t>(o) & (4 * sizeof(TOut) - 1)) == 0;
    const int n4 = hidden >> 2;
    float4 v[kVec];
    double ss = 0.0;
    if (vec) {
#pragma unroll
        for (int k = 0; k < kVec; ++k) {
            const int i4 = threadIdx.x + 256 * k;
            v[k] = i4 < n4 ? reinterpret_cast<const float4 *>(xr)[i4] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (fold.n > 0) {   // the residual's pending split-K partials, in slice order, written back
#pragma unroll
            for (int k = 0; k < kVec; ++k) {
                const int i4 = threadIdx.x + 256 * k;
                if (i4 < n4) {
                    for (int sl = 0; sl < fold.n; ++sl) {
                        const float4 a = reinterpret_cast<const float4 *>(fold.slices + sl * fold.stride + xrow)[i4];
                        v[k].x += a.x; v[k].y += a.y; v[k].z += a.z; v[k].w += a.w;
                    }
                    reinterpret_cast<float4 *>(xr)[i4] = v[k];
                }
            }
        }
#pragma unroll
        for (int k = 0; k < kVec; ++k)
            ss += static_cast<double>(v[k].x) * v[k].x + static_cast<double>(v[k].y) * v[k].y +
                  static_cast<double>(v[k].z) * v[k].z + static_cast<double>(v[k].w) * v[k].w;
    } else {
        for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
            float xv = xr[i];
            if (fold.n > 0) {
                for (int sl = 0; sl < fold.n; ++sl) xv += fold.slices[sl * fold.stride + xrow + i];
                xr[i] = xv;
            }
            ss += static_cast<double>(xv) * xv;
        }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    __shared__ double part[8];
    __shared__ float s_scale;
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) t += part[k];
        const double ms = t / static_cast<double>(hidden);
        s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(ms), eps)));
    }
    __syncthreads();
    const float scale = s_scale;
    if (vec) {
#pragma unroll
        for (int k = 0; k < kVec; ++k) {
            const int i4 = threadIdx.x + 256 * k;
            if (i4 < n4) {
                const float4 wv = reinterpret_cast<const float4 *>(w)[i4];
                put4<TOut>(o + 4 * i4, make_float4(__fmul_rn(__fmul_rn(v[k].x, scale), wv.x),
                                                   __fmul_rn(__fmul_rn(v[k].y, scale), wv.y),
                                                   __fmul_rn(__fmul_rn(v[k].z, scale), wv.z),
                                                   __fmul_rn(__fmul_rn(v[k].w, scale), wv.w)));
            }
        }
    } else {
        for (int i = threadIdx.x; i < hidden; i += blockDim.x) put<TOut>(o + i, __fmul_rn(__fmul_rn(xr[i], scale), w[i]));
    }
}

// x[r] += the pending split-K slices of row r, in slice order (for readers
// of the residual other than the RMSNorms, which fold as they read).
__global__ void __launch_bounds__(256) residual_fold_kernel(float *x, int hidden, ResidualFold fold) {
    pdl_trigger();
    pdl_wait();
    const size_t row = static_cast<size_t>(blockIdx.x) * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        float v = x[row + i];
        for (int sl = 0; sl < fold.n; ++sl) v += fold.slices[sl * fold.stride + row + i];
        x[row + i] = v;
    }
}

template <typename TW>
__global__ void embed_kernel(const int *ids, const TW *embd, int hidden, int vocab, float *x, DevError *err) {
    pdl_trigger();
    pdl_wait();   // everything below reads or writes memory of earlier kernels
    const int r = blockIdx.x;
    const int id = ids[r];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) report_error(err, kErrRowBounds, kWhereEmbed, r, id);
        return;
    }
    const TW *src = embd + static_cast<size_t>(id) * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        if constexpr (sizeof(TW) == 4) x[static_cast<size_t>(r) * hidden + i] = src[i];
        else x[static_cast<size_t>(r) * hidden + i] = __bfloat162float(src[i]);
    }
}

// Audio projector LayerNorm (audio-encoder.cpp:399-407 / 851: mean and
// variance over the row, eps 1e-5, times weight plus bias), one CTA per row;
// mean and variance accumulated in double, two passes over the row.
template <typename TOut>
__global__ void __launch_bounds__(256) layernorm_kernel(const float *x, int width, const float *w, const float *b,
                                                        float eps, TOut *out) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    const float *xr = x + static_cast<size_t>(r) * width;
    __shared__ double part[8];
    __shared__ float s_mean, s_scale;
    double acc = 0.0;
    for (int i = threadIdx.x; i < width; i += blockDim.x) acc += xr[i];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) t += part[k];
        s_mean = static_cast<float>(t / width);
    }
    __syncthreads();
    const float mean = s_mean;
    acc = 0.0;
    for (int i = threadIdx.x; i < width; i += blockDim.x) {
        const double d = static_cast<double>(xr[i]) - mean;
        acc += d * d;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) t += part[k];
        s_scale = static_cast<float>(1.0 / sqrt(t / width + static_cast<double>(eps)));
    }
    __syncthreads();
    const float scale = s_scale;
    TOut *o = out + static_cast<size_t>(r) * width;
    for (int i = threadIdx.x; i < width; i += blockDim.x) put<TOut>(o + i, (xr[i] - mean) * scale * w[i] + b[i]);
}

// out[r][j] = act(c[r][j] + bias[j]) with act = GELU (erf form,
// 0.5 x (1 + erf(x / sqrt 2)), as the projector's ggml_gelu_erf) or identity.
template <typename TOut>
__global__ void bias_act_kernel(const float *c, const float *bias, int n, int width, int gelu, TOut *out) {
    pdl_trigger();
    pdl_wait();
    const size_t total = static_cast<size_t>(n) * width;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        float v = c[i] + bias[i % width];
        if (gelu) v = 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
        put<TOut>(out + i, v);
    }
}

// Decoder input (the device side of src/decoder-input.cpp:64-98): row t is
// the embedding row of ids[t], or, where src[t] >= 0, audio row src[t]
// (rows[src[t]] points at its hidden f32 values).  One CTA per row, 16-byte
// copies when hidden is a multiple of 4; ids and src were checked on the host.
template <typename TW>
__global__ void decoder_input_kernel(const int *ids, const int *src, const TW *embd, int hidden,
                                     const float *const *rows, float *x) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x;
    float *dst = x + static_cast<size_t>(t) * hidden;
    const int a = src[t];
    if (a >= 0) {
        const float *s = rows[a];
        if ((hidden & 3) == 0 && (reinterpret_cast<uintptr_t>(s) & 15) == 0) {
            for (int i = threadIdx.x; i < (hidden >> 2); i += blockDim.x)
                reinterpret_cast<float4 *>(dst)[i] = reinterpret_cast<const float4 *>(s)[i];
        } else {
            for (int i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = s[i];
        }
        return;
    }
    const TW *e = embd + static_cast<size_t>(ids[t]) * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        if constexpr (sizeof(TW) == 4) dst[i] = e[i];
        else dst[i] = __bfloat162float(e[i]);
    }
}

// Four consecutive elements -> float4.
template <typename T> __device__ __forceinline__ float4 ld4(const T *p);
template <> __device__ __forceinline__ float4 ld4<float>(const float *p) { return *reinterpret_cast<const float4 *>(p); }
template <> __device__ __forceinline__ float4 ld4<__nv_bfloat16>(const __nv_bfloat16 *p) {
    const uint2 w = *reinterpret_cast<const uint2 *>(p);
    return make_float4(bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y));
}

// SIMT tiled GEMM: 64 (m) x 64 (n) tile, BK = 16, 256 threads, 4x4 per
// thread, optional split-K over gridDim.z (atomic accumulate).
constexpr int BM = 64, BN = 64, BK = 16, PAD = 4;

template <typename TX, typename TW>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const TX *X, const TW *W, float *C, int M, int N, int K,
                                                        int k_per_split, int atomic_out) {
    pdl_trigger();
    pdl_wait();   // everything below reads or writes memory of earlier kernels
    __shared__ __align__(16) float As[BK][BM + PAD];
    __shared__ __align__(16) float Bs[BK][BN + PAD];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int kb = blockIdx.z * k_per_split;
    const int ke = min(K, kb + k_per_split);
    const int lr = tid >> 2, lk = (tid & 3) * 4;   // loader: row within tile, k offset
    const int tx = tid & 15, ty = tid >> 4;
    float acc[4][4] = {};
    const bool xm = (m0 + lr) < M, wn = (n0 + lr) < N;
    const TX *xp = X + static_cast<size_t>(m0 + lr) * K + lk;
    const TW *wp = W + static_cast<size_t>(n0 + lr) * K + lk;
    float4 xa = make_float4(0.f, 0.f, 0.f, 0.f), wa = xa;
    if (kb < ke) {
        if (xm) xa = ld4<TX>(xp + kb);
        if (wn) wa = ld4<TW>(wp + kb);
    }
    for (int k0 = kb; k0 < ke; k0 += BK) {
        As[lk + 0][lr] = xa.x; As[lk + 1][lr] = xa.y; As[lk + 2][lr] = xa.z; As[lk + 3][lr] = xa.w;
        Bs[lk + 0][lr] = wa.x; Bs[lk + 1][lr] = wa.y; Bs[lk + 2][lr] = wa.z; Bs[lk + 3][lr] = wa.w;
        __syncthreads();
        if (k0 + BK < ke) {
            if (xm) xa = ld4<TX>(xp + k0 + BK);
            if (wn) wa = ld4<TW>(wp + k0 + BK);
        }
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            const float4 a = *reinterpret_cast<const float4 *>(&As[k][ty * 4]);
            const float4 b = *reinterpret_cast<const float4 *>(&Bs[k][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w};
            const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int jn = 0; jn < 4; ++jn) acc[i][jn] = fmaf(av[i], bv[jn], acc[i][jn]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int jn = 0; jn < 4; ++jn) {
            const int n = n0 + tx * 4 + jn;
            if (n >= N) continue;
            float *c = C + static_cast<size_t>(m) * N + n;
            if (atomic_out) atomicAdd(c, acc[i][jn]);
            else *c = acc[i][jn];
        }
    }
}

// Small-M path (M <= 4): one warp per output column n, lanes stride over K,
// X rows staged in shared memory as f32.
template <typename TX, typename TW, int MM>
__global__ void __launch_bounds__(256) gemv_kernel(const TX *X, const TW *W, float *C, int M, int N, int K,
                                                   int accumulate) {
    pdl_trigger();
    pdl_wait();   // everything below reads or writes memory of earlier kernels
    extern __shared__ __align__(16) float xs[];   // [MM][K]
    for (int e = threadIdx.x * 4; e < M * K; e += blockDim.x * 4) {
        const float4 v = ld4<TX>(X + e);
        *reinterpret_cast<float4 *>(xs + e) = v;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * 8 + warp;
    if (n >= N) return;
    const TW *w = W + static_cast<size_t>(n) * K;
    float acc[MM] = {};
    for (int k = lane * 4; k < K; k += 128) {
        const float4 wv = ld4<TW>(w + k);
#pragma unroll
        for (int m = 0; m < MM; ++m) {
            if (m < M) {
                const float4 xv = *reinterpret_cast<const float4 *>(xs + m * K + k);
                acc[m] = fmaf(wv.x, xv.x, acc[m]);
                acc[m] = fmaf(wv.y, xv.y, acc[m]);
                acc[m] = fmaf(wv.z, xv.z, acc[m]);
                acc[m] = fmaf(wv.w, xv.w, acc[m]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < MM; ++m) {
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
    }
    if (lane == 0) {
#pragma unroll
        for (int m = 0; m < MM; ++m) {
            if (m < M) {
                float *c = C + static_cast<size_t>(m) * N + n;
                *c = accumulate ? *c + acc[m] : acc[m];
            }
        }
    }
}

template <typename TOut>
__global__ void swiglu_kernel(const float *gu, int M, int F, TOut *out) {
    pdl_trigger();
    pdl_wait();   // everything below reads or writes memory of earlier kernels
    const size_t total = static_cast<size_t>(M) * F;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        // gu rows hold gate and up interleaved one by one: [g0 u0 g1 u1 ...].
        const size_t m = i / F, jf = i % F;
        const float2 gv = *reinterpret_cast<const float2 *>(gu + m * 2 * F + 2 * jf);
        const float g = gv.x, u = gv.y;
        const float s = g / (1.0f + expf(-g));
        put<TOut>(out + i, s * u);
    }
}

// Rows to e4m3 codes with one f32 scale per row (amax / 448, 1 for an all-zero
// row): the token operand of the FP8 projections, and the weights at load.
// One CTA per row; the row's values are built once into shared memory:
//   kQ8Rows:    bf16 input rows [n][K]
//   kQ8RmsNorm: RMSNorm of f32 rows x [n][K] with weights w (the formula of
//               rmsnorm_kernel, double sum of squares)
//   kQ8SwiGLU:  silu(gate) * up of f32 rows gu [n][2K], gate and up
//               interleaved one by one (as swiglu_kernel reads)
enum Q8Mode { kQ8Rows = 0, kQ8RmsNorm = 1, kQ8SwiGLU = 2 };
constexpr int kQ8Threads = 256;
constexpr int kQ8MaxVec = 6;   // float4 groups per thread: rows up to 256 x 6 x 4 = 6144 wide

// The row stays in registers (kQ8MaxVec groups of 4 per thread, 16-byte
// loads); K % 4 == 0 (checked at launch).
template <int MODE>
__global__ void __launch_bounds__(kQ8Threads) rows_q8_kernel(const void *in, int K, const float *w, float eps,
                                                             uint8_t *out, float *scales, ResidualFold fold) {
    pdl_trigger();
    pdl_wait();   // the input rows come from the kernels before this one
    __shared__ double dpart[kQ8Threads / 32];
    __shared__ float fpart[kQ8Threads / 32];
    __shared__ float s_val;
    const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k4 = K >> 2;
    float4 v[kQ8MaxVec];
#pragma unroll
    for (int g = 0; g < kQ8MaxVec; ++g) {
        const int i4 = threadIdx.x + kQ8Threads * g;
        v[g] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i4 < k4) {
            if constexpr (MODE == kQ8Rows) {
                const uint2 b = reinterpret_cast<const uint2 *>(static_cast<const __nv_bfloat16 *>(in) +
                                                                static_cast<size_t>(r) * K)[i4];
                v[g] = make_float4(bf16lo(b.x), bf16hi(b.x), bf16lo(b.y), bf16hi(b.y));
            } else if constexpr (MODE == kQ8RmsNorm) {
                float4 *xr = reinterpret_cast<float4 *>(const_cast<float *>(static_cast<const float *>(in)) +
                                                        static_cast<size_t>(r) * K);
                v[g] = xr[i4];
                if (fold.n > 0) {   // the residual's pending split-K partials, in slice order, written back
                    for (int sl = 0; sl < fold.n; ++sl) {
                        const float4 a = reinterpret_cast<const float4 *>(fold.slices + sl * fold.stride +
                                                                          static_cast<size_t>(r) * K)[i4];
                        v[g].x += a.x; v[g].y += a.y; v[g].z += a.z; v[g].w += a.w;
                    }
                    xr[i4] = v[g];
                }
            } else {
                // gate and up interleaved one by one: features 4 i4 .. 4 i4 + 3 are 8 floats
                const float *gp = static_cast<const float *>(in) + static_cast<size_t>(r) * 2 * K + 8 * i4;
                const float4 a = *reinterpret_cast<const float4 *>(gp);
                const float4 b = *reinterpret_cast<const float4 *>(gp + 4);
                const float4 gv = make_float4(a.x, a.z, b.x, b.z), uv = make_float4(a.y, a.w, b.y, b.w);
                v[g] = make_float4(gv.x / (1.0f + expf(-gv.x)) * uv.x, gv.y / (1.0f + expf(-gv.y)) * uv.y,
                                   gv.z / (1.0f + expf(-gv.z)) * uv.z, gv.w / (1.0f + expf(-gv.w)) * uv.w);
            }
        }
    }
    if constexpr (MODE == kQ8RmsNorm) {
        // RMSNorm as rmsnorm_kernel: double sum of squares, then x * scale * w rounded per op
        double ss = 0.0;
#pragma unroll
        for (int g = 0; g < kQ8MaxVec; ++g)
            ss += static_cast<double>(v[g].x) * v[g].x + static_cast<double>(v[g].y) * v[g].y +
                  static_cast<double>(v[g].z) * v[g].z + static_cast<double>(v[g].w) * v[g].w;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) dpart[warp] = ss;
        __syncthreads();
        if (threadIdx.x == 0) {
            double t = 0.0;
            for (int k = 0; k < kQ8Threads / 32; ++k) t += dpart[k];
            s_val = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(t / static_cast<double>(K)), eps)));
        }
        __syncthreads();
        const float sc = s_val;
#pragma unroll
        for (int g = 0; g < kQ8MaxVec; ++g) {
            const int i4 = threadIdx.x + kQ8Threads * g;
            if (i4 < k4) {
                const float4 wv = reinterpret_cast<const float4 *>(w)[i4];
                v[g] = make_float4(__fmul_rn(__fmul_rn(v[g].x, sc), wv.x), __fmul_rn(__fmul_rn(v[g].y, sc), wv.y),
                                   __fmul_rn(__fmul_rn(v[g].z, sc), wv.z), __fmul_rn(__fmul_rn(v[g].w, sc), wv.w));
            }
        }
    }
    float amax = 0.0f;
#pragma unroll
    for (int g = 0; g < kQ8MaxVec; ++g)
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[g].x), fabsf(v[g].y)), fmaxf(fabsf(v[g].z), fabsf(v[g].w))));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) fpart[warp] = amax;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = 0.0f;
        for (int k = 0; k < kQ8Threads / 32; ++k) m = fmaxf(m, fpart[k]);
        const float sc = m > 0.0f ? __fdiv_rn(m, kE4m3Max) : 1.0f;
        scales[r] = sc;
        s_val = m > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
    }
    __syncthreads();
    const float inv = s_val;
    uint32_t *o = reinterpret_cast<uint32_t *>(out + static_cast<size_t>(r) * K);
#pragma unroll
    for (int g = 0; g < kQ8MaxVec; ++g) {
        const int i4 = threadIdx.x + kQ8Threads * g;
        if (i4 < k4)
            o[i4] = static_cast<uint32_t>(f_to_e4m3(v[g].x * inv)) | (static_cast<uint32_t>(f_to_e4m3(v[g].y * inv)) << 8) |
                    (static_cast<uint32_t>(f_to_e4m3(v[g].z * inv)) << 16) |
                    (static_cast<uint32_t>(f_to_e4m3(v[g].w * inv)) << 24);
    }
}

// Split argmax: CTA (r, s) scans slice s of row r (16-byte loads when the
// row allows them) and writes its (max, index) partial; the last CTA of the
// row to finish (per-row counter, which it resets) merges the partials in
// slice order.  The first maximum wins (ties keep the smaller index); NaN never wins.
__device__ __forceinline__ void take_max(float v, int i, float &best, int &idx) {
    if (v > best || (v == best && i >= 0 && (idx < 0 || i < idx))) {
        best = v;
        idx = i;
    }
}

__device__ __forceinline__ void block_max(float &best, int &idx, float *sb, int *si) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        take_max(ob, oi, best, idx);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sb[warp] = best;
        si[warp] = idx;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? sb[lane] : -INFINITY;
        idx = lane < nw ? si[lane] : -1;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            take_max(ob, oi, best, idx);
        }
    }
}

__global__ void __launch_bounds__(512) argmax_split_kernel(const float *logits, int V, int S, float *part_v,
                                                           int *part_i, int *counters, int *ids) {
    pdl_trigger();
    pdl_wait();   // everything below reads or writes memory of earlier kernels
    const int r = blockIdx.x, sl = blockIdx.y;
    const float *row = logits + static_cast<size_t>(r) * V;
    float best = -INFINITY;
    int idx = -1;
    if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
        const int v4 = V >> 2, ch = (v4 + S - 1) / S;
        const int lo = sl * ch, hi = min(v4, lo + ch);
        for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            const float4 q = reinterpret_cast<const float4 *>(row)[i];
            if (q.x > best) { best = q.x; idx = 4 * i; }
            if (q.y > best) { best = q.y; idx = 4 * i + 1; }
            if (q.z > best) { best = q.z; idx = 4 * i + 2; }
            if (q.w > best) { best = q.w; idx = 4 * i + 3; }
        }
    } else {
        const int ch = (V + S - 1) / S;
        const int lo = sl * ch, hi = min(V, lo + ch);
        for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            const float v = row[i];
            if (v > best) { best = v; idx = i; }
        }
    }
    __shared__ float sb[32];
    __shared__ int si[32];
    __shared__ int last;
    block_max(best, idx, sb, si);
    if (threadIdx.x == 0) {
        if (S == 1) {
            ids[r] = idx;
            last = 0;
        } else {
            part_v[r * S + sl] = best;
            part_i[r * S + sl] = idx;
            __threadfence();
            last = atomicAdd(&counters[r], 1) == S - 1;
        }
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    __threadfence();
    float b = -INFINITY;
    int bi = -1;
    for (int k = 0; k < S; ++k) take_max(__ldcg(part_v + r * S + k), __ldcg(part_i + r * S + k), b, bi);
    ids[r] = bi;
    counters[r] = 0;
}

// Largest row norm of a bf16 weight matrix [rows][H] (warp per row), for the
// error bound of argmax_refine_kernel.  *out must start at 0; row norms are
// positive, so their float bits order like the floats.
__global__ void __launch_bounds__(256) row_norm_max_kernel(const __nv_bfloat16 *W, int rows, int H, float *out) {
    const int lane = threadIdx.x & 31;
    const int warps = static_cast<int>(gridDim.x * (blockDim.x >> 5));
    for (int r = static_cast<int>(blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)); r < rows; r += warps) {
        const __nv_bfloat16 *w = W + static_cast<size_t>(r) * H;
        double ss = 0.0;
        for (int k = lane; k < H; k += 32) {
            const double v = __bfloat162float(w[k]);
            ss += v * v;
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) atomicMax(reinterpret_cast<int *>(out), __float_as_int(static_cast<float>(sqrt(ss)) * 1.0001f));
    }
}

// Exact re-scoring of the greedy argmax behind the bf16 LM head.  The head
// GEMM multiplies bf16 weights by the bf16-rounded final hidden row b =
// bf16(h), so an approximate logit a_j differs from the f32 logit
// l_j = sum_k W_jk h_k by at most
//     sum_k |W_jk| |h_k - b_k| + (f32 accumulation) <= (2^-8 + 2^-12) ||W_j|| ||h||
//     <= e = (2^-8 + 2^-12) wmax ||h||                 (Cauchy-Schwarz; wmax = max_j ||W_j||).
// The f32 argmax j* therefore has a_j* >= l_j* - e >= l_jmax - e >= a_jmax - 2e:
// every token whose approximate logit is within 2e of the approximate maximum
// is re-scored exactly (bf16 weight row x f32 h, f32 accumulation), and the
// row's id becomes the first maximum of those scores, i.e. the argmax of the
// f32 logits (as text-decoder.cpp:2266-2274 takes it over its f32 logits).
// Grid (rows, slices): each CTA rebuilds h from the residual row exactly as
// rmsnorm_kernel does, scans its slice, and a warp re-scores each candidate;
// scores meet in a per-row 64-bit key (ordered float bits, then the inverted
// index so that the lower index wins a tie), and the row's last CTA writes the
// id and resets the key and counter.
__global__ void __launch_bounds__(256) argmax_refine_kernel(const float *logits, int V, int S, const float *x,
                                                            const int *rows, int H, const float *norm_w, float eps,
                                                            const __nv_bfloat16 *W, const float *wmax,
                                                            unsigned long long *keys, int *counters, int *ids) {
    pdl_trigger();
    pdl_wait();   // ids and logits come from the kernels before this one
    extern __shared__ __align__(16) float hs[];   // [H]
    __shared__ double part[8];
    __shared__ float s_scale, s_thr;
    __shared__ int last;
    const int r = blockIdx.x, sl = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *xr = x + static_cast<size_t>(rows ? rows[r] : r) * H;
    double ss = 0.0;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ss += static_cast<double>(xr[i]) * xr[i];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) part[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) t += part[k];
        s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(t / static_cast<double>(H)), eps)));
    }
    __syncthreads();
    const float scale = s_scale;
    double hh = 0.0;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float v = __fmul_rn(__fmul_rn(xr[i], scale), norm_w[i]);
        hs[i] = v;
        hh += static_cast<double>(v) * v;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) hh += __shfl_xor_sync(0xffffffffu, hh, o);
    __syncthreads();   // part[] is reused below
    if (lane == 0) part[warp] = hh;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) t += part[k];
        const double e = (1.0 / 256.0 + 1.0 / 4096.0) * static_cast<double>(*wmax) * sqrt(t);
        const float amax = logits[static_cast<size_t>(r) * V + ids[r]];
        s_thr = static_cast<float>(static_cast<double>(amax) - 2.0 * e * 1.01);
    }
    __syncthreads();
    const float thr = s_thr;
    const float *row = logits + static_cast<size_t>(r) * V;
    // Exact f32 score of token jj by the whole warp, merged into the row's key.
    auto rescore = [&](int jj) {
        const __nv_bfloat16 *w = W + static_cast<size_t>(jj) * H;
        float acc = 0.0f;
        for (int k = lane * 8; k < H; k += 256) {   // H % 8 == 0 (checked at launch)
            const uint4 q = *reinterpret_cast<const uint4 *>(w + k);
            acc = fmaf(bf16lo(q.x), hs[k + 0], acc); acc = fmaf(bf16hi(q.x), hs[k + 1], acc);
            acc = fmaf(bf16lo(q.y), hs[k + 2], acc); acc = fmaf(bf16hi(q.y), hs[k + 3], acc);
            acc = fmaf(bf16lo(q.z), hs[k + 4], acc); acc = fmaf(bf16hi(q.z), hs[k + 5], acc);
            acc = fmaf(bf16lo(q.w), hs[k + 6], acc); acc = fmaf(bf16hi(q.w), hs[k + 7], acc);
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
            const uint32_t u = __float_as_uint(acc);
            const uint32_t ou = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
            atomicMax(keys + r, (static_cast<unsigned long long>(ou) << 32) | (0xffffffffu - static_cast<uint32_t>(jj)));
        }
    };
    const int nwarps = static_cast<int>(blockDim.x >> 5);
    if ((V & 3) == 0) {
        // Slices of whole float4 groups; a warp takes 128 groups (512 logits) per
        // pass, four independent 16-byte loads per lane in flight at once.
        const int v4 = V >> 2, ch4 = (v4 + S - 1) / S;
        const int lo4 = sl * ch4, hi4 = min(v4, lo4 + ch4);
        const float4 *row4 = reinterpret_cast<const float4 *>(row);
        for (int c0 = lo4 + warp * 128; c0 < hi4; c0 += nwarps * 128) {
            float4 a[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int idx = c0 + u * 32 + lane;
                a[u] = idx < hi4 ? row4[idx] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            }
            uint32_t m = 0;   // bit 4u + c: component c of group u is a candidate
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                m |= (a[u].x >= thr ? 1u : 0u) << (4 * u);
                m |= (a[u].y >= thr ? 1u : 0u) << (4 * u + 1);
                m |= (a[u].z >= thr ? 1u : 0u) << (4 * u + 2);
                m |= (a[u].w >= thr ? 1u : 0u) << (4 * u + 3);
            }
            unsigned who = __ballot_sync(0xffffffffu, m != 0);
            while (who) {
                const int src = __ffs(who) - 1;
                who &= who - 1;
                uint32_t mm = __shfl_sync(0xffffffffu, m, src);
                while (mm) {
                    const int b = __ffs(mm) - 1;
                    mm &= mm - 1;
                    rescore(4 * (c0 + (b >> 2) * 32 + src) + (b & 3));
                }
            }
        }
    } else {
        const int ch = (V + S - 1) / S;
        const int lo = sl * ch, hi = min(V, lo + ch);
        for (int base = lo + warp * 32; base < hi; base += nwarps * 32) {
            const int j = base + lane;
            unsigned mask = __ballot_sync(0xffffffffu, j < hi && row[j] >= thr);
            while (mask) {
                const int jj = base + __ffs(mask) - 1;
                mask &= mask - 1;
                rescore(jj);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(&counters[r], 1) == S - 1;
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    __threadfence();
    const unsigned long long key = atomicExch(keys + r, 0ull);
    if (key != 0ull) ids[r] = static_cast<int>(0xffffffffu - static_cast<uint32_t>(key & 0xffffffffull));
    counters[r] = 0;
}

// GGUF tensor bytes (f32 / f16 / bf16) -> device weight dtype (f32 / bf16, RNE).
template <typename TD>
__global__ void convert_kernel(const void *src, int src_type, TD *dst, size_t n) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        float v;
        if (src_type == 0) v = static_cast<const float *>(src)[i];
        else if (src_type == 1) v = __half2float(static_cast<const __half *>(src)[i]);
        else v = __bfloat162float(static_cast<const __nv_bfloat16 *>(src)[i]);
        put<TD>(dst + i, v);
    }
}

int g_num_sms = 148;

}  // namespace

cudaError_t launch_convert(const void *src, int src_ggml_type, void *dst, int dst_dtype, size_t n, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const int blocks = static_cast<int>((n + 255) / 256 < 8192 ? (n + 255) / 256 : 8192);
    if (dst_dtype == kActF32) convert_kernel<float><<<blocks, 256, 0, st>>>(src, src_ggml_type, static_cast<float *>(dst), n);
    else convert_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(src, src_ggml_type, static_cast<__nv_bfloat16 *>(dst), n);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(float *x, const int *rows, int n, int hidden, const float *w, float eps, void *out,
                           int out_dtype, cudaStream_t st, ResidualFold fold) {
    if (n <= 0) return cudaSuccess;
    if (fold.n > 0 && (hidden & 3) != 0) return cudaErrorInvalidValue;
    if (out_dtype == kActF32)
        return launch_pdl(rmsnorm_kernel<float>, dim3(n), dim3(256), 0, st, x, rows, hidden, w, eps,
                          static_cast<float *>(out), fold);
    return launch_pdl(rmsnorm_kernel<__nv_bfloat16>, dim3(n), dim3(256), 0, st, x, rows, hidden, w, eps,
                      static_cast<__nv_bfloat16 *>(out), fold);
}

cudaError_t launch_residual_fold(float *x, int n, int hidden, ResidualFold fold, cudaStream_t st) {
    if (n <= 0 || fold.n <= 0) return cudaSuccess;
    return launch_pdl(residual_fold_kernel, dim3(n), dim3(256), 0, st, x, hidden, fold);
}

cudaError_t launch_layernorm(const float *x, int n, int width, const float *w, const float *b, float eps, void *out,
                             int out_dtype, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (out_dtype == kActF32)
        return launch_pdl(layernorm_kernel<float>, dim3(n), dim3(256), 0, st, x, width, w, b, eps,
                          static_cast<float *>(out));
    return launch_pdl(layernorm_kernel<__nv_bfloat16>, dim3(n), dim3(256), 0, st, x, width, w, b, eps,
                      static_cast<__nv_bfloat16 *>(out));
}

cudaError_t launch_bias_act(const float *c, const float *bias, int n, int width, bool gelu, void *out, int out_dtype,
                            cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const size_t total = static_cast<size_t>(n) * width;
    const unsigned blocks = static_cast<unsigned>(std::min<size_t>((total + 255) / 256, 65535));
    if (out_dtype == kActF32)
        return launch_pdl(bias_act_kernel<float>, dim3(blocks), dim3(256), 0, st, c, bias, n, width, gelu ? 1 : 0,
                          static_cast<float *>(out));
    return launch_pdl(bias_act_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st, c, bias, n, width,
                      gelu ? 1 : 0, static_cast<__nv_bfloat16 *>(out));
}

cudaError_t launch_decoder_input(const int *ids, const int *src, int n, const void *embd, int w_dtype, int hidden,
                                 const float *const *rows, float *x, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (w_dtype == kActF32)
        return launch_pdl(decoder_input_kernel<float>, dim3(n), dim3(256), 0, st, ids, src,
                          static_cast<const float *>(embd), hidden, rows, x);
    return launch_pdl(decoder_input_kernel<__nv_bfloat16>, dim3(n), dim3(256), 0, st, ids, src,
                      static_cast<const __nv_bfloat16 *>(embd), hidden, rows, x);
}

cudaError_t launch_embed(const int *ids, int n, const void *embd, int w_dtype, int hidden, int vocab, float *x,
                         DevError *err, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (w_dtype == kActF32)
        return launch_pdl(embed_kernel<float>, dim3(n), dim3(256), 0, st, ids, static_cast<const float *>(embd), hidden, vocab,
                          x, err);
    return launch_pdl(embed_kernel<__nv_bfloat16>, dim3(n), dim3(256), 0, st, ids,
                      static_cast<const __nv_bfloat16 *>(embd), hidden, vocab, x, err);
}

template <typename TX, typename TW>
static cudaError_t gemm_t(const TX *X, const TW *W, float *C, int M, int N, int K, int epilogue, cudaStream_t st) {
    if (M <= 4) {
        const size_t sm = static_cast<size_t>(M) * K * sizeof(float);   // opted in by prepare_dense
        return launch_pdl(gemv_kernel<TX, TW, 4>, dim3((N + 7) / 8), dim3(256), sm, st, X, W, C, M, N, K, epilogue);
    }
    const int tm = (M + BM - 1) / BM, tn = (N + BN - 1) / BN;
    int splits = 1;
    const int want = 2 * g_num_sms;
    if (tm * tn < want) {
        splits = (want + tm * tn - 1) / (tm * tn);
        const int max_splits = K / 256 > 0 ? K / 256 : 1;
        if (splits > max_splits) splits = max_splits;
    }
    int kps = (K + splits - 1) / splits;
    kps = (kps + BK - 1) / BK * BK;
    splits = (K + kps - 1) / kps;
    const bool atomic = splits > 1 || epilogue == 1;
    if (splits > 1 && epilogue == 0) {
        cudaError_t e = cudaMemsetAsync(C, 0, static_cast<size_t>(M) * N * sizeof(float), st);
        if (e != cudaSuccess) return e;
    }
    dim3 grid(tn, tm, splits);
    return launch_pdl(gemm_simt_kernel<TX, TW>, grid, dim3(256), 0, st, X, W, C, M, N, K, kps, atomic ? 1 : 0);
}

cudaError_t prepare_dense(int max_k) {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
        sms > 0)
        g_num_sms = sms;
    const int sm = 4 * max_k * static_cast<int>(sizeof(float));
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<float, float, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm)) != cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<__nv_bfloat16, __nv_bfloat16, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm)) !=
        cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<float, __nv_bfloat16, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm)) !=
        cudaSuccess)
        return e;
    return cudaFuncSetAttribute(gemv_kernel<__nv_bfloat16, float, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
}

cudaError_t launch_gemm(const void *X, int x_dtype, const void *W, int w_dtype, float *C, int M, int N, int K,
                        int epilogue, cudaStream_t st) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (K % BK != 0) return cudaErrorInvalidValue;
    if (x_dtype == kActF32 && w_dtype == kActF32)
        return gemm_t(static_cast<const float *>(X), static_cast<const float *>(W), C, M, N, K, epilogue, st);
    if (x_dtype == kActBF16 && w_dtype == kActBF16)
        return gemm_t(static_cast<const __nv_bfloat16 *>(X), static_cast<const __nv_bfloat16 *>(W), C, M, N, K, epilogue, st);
    if (x_dtype == kActF32 && w_dtype == kActBF16)
        return gemm_t(static_cast<const float *>(X), static_cast<const __nv_bfloat16 *>(W), C, M, N, K, epilogue, st);
    return gemm_t(static_cast<const __nv_bfloat16 *>(X), static_cast<const float *>(W), C, M, N, K, epilogue, st);
}

cudaError_t launch_swiglu(const float *gu, int M, int F, void *out, int out_dtype, cudaStream_t st) {
    if (M <= 0) return cudaSuccess;
    const size_t total = static_cast<size_t>(M) * F;
    const int blocks = static_cast<int>((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
    if (out_dtype == kActF32)
        return launch_pdl(swiglu_kernel<float>, dim3(blocks), dim3(256), 0, st, gu, M, F, static_cast<float *>(out));
    return launch_pdl(swiglu_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st, gu, M, F,
                      static_cast<__nv_bfloat16 *>(out));
}

cudaError_t launch_rows_q8(int mode, const void *in, int n, int K, const float *w, float eps, void *out, float *scales,
                           cudaStream_t st, ResidualFold fold) {
    if (n <= 0) return cudaSuccess;
    if (K <= 0 || K % 4 != 0 || K > kQ8Threads * kQ8MaxVec * 4) return cudaErrorInvalidValue;
    uint8_t *o = static_cast<uint8_t *>(out);
    switch (mode) {
        case kQ8Rows:
            return launch_pdl(rows_q8_kernel<kQ8Rows>, dim3(n), dim3(kQ8Threads), 0, st, in, K, w, eps, o, scales,
                              ResidualFold{});
        case kQ8RmsNorm:
            return launch_pdl(rows_q8_kernel<kQ8RmsNorm>, dim3(n), dim3(kQ8Threads), 0, st, in, K, w, eps, o, scales,
                              fold);
        case kQ8SwiGLU:
            return launch_pdl(rows_q8_kernel<kQ8SwiGLU>, dim3(n), dim3(kQ8Threads), 0, st, in, K, w, eps, o, scales,
                              ResidualFold{});
        default: return cudaErrorInvalidValue;
    }
}

int rows_q8_max_k() { return kQ8Threads * kQ8MaxVec * 4; }

cudaError_t launch_argmax_split(const float *logits, int M, int V, int *ids, float *part_v, int *part_i,
                                int *counters, int max_slices, int num_sms, cudaStream_t st) {
    if (M <= 0) return cudaSuccess;
    int S = (2 * num_sms + M - 1) / M;
    if (S > max_slices) S = max_slices;
    if (S > (V + 4095) / 4096) S = (V + 4095) / 4096;   // slices of at least ~4K logits
    if (S < 1) S = 1;
    return launch_pdl(argmax_split_kernel, dim3(M, S), dim3(512), 0, st, logits, V, S, part_v, part_i, counters,
                      ids);
}

cudaError_t launch_row_norm_max(const void *W, int rows, int H, float *out, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float), st);
    if (e != cudaSuccess) return e;
    const int blocks = (rows + 7) / 8 < 4096 ? (rows + 7) / 8 : 4096;
    row_norm_max_kernel<<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16 *>(W), rows, H, out);
    return cudaGetLastError();
}

cudaError_t launch_argmax_refine(const float *logits, int M, int V, const float *x, const int *rows, int H,
                                 const float *norm_w, float eps, const void *W, const float *wmax,
                                 unsigned long long *keys, int *counters, int *ids, int num_sms, cudaStream_t st) {
    if (M <= 0) return cudaSuccess;
    if (H % 8 != 0 || H > 12 * 1024) return cudaErrorInvalidValue;
    int S = (2 * num_sms + M - 1) / M;
    if (S > 64) S = 64;
    if (S > (V + 4095) / 4096) S = (V + 4095) / 4096;
    if (S < 1) S = 1;
    return launch_pdl(argmax_refine_kernel, dim3(M, S), dim3(256), static_cast<size_t>(H) * sizeof(float), st, logits,
                      V, S, x, rows, H, norm_w, eps, static_cast<const __nv_bfloat16 *>(W), wmax, keys, counters, ids);
}

}  // namespace qkv
