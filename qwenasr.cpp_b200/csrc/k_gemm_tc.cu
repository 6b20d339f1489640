// Tensor-core projections on sm_100a: C[M][N] (+)= X[M][K] . W[N][K]^T with
// bf16 X and W, f32 accumulation in TMEM (tcgen05.mma kind::f16), operands
// staged by TMA (cp.async.bulk.tensor, 128-byte swizzle, no multicast).
// Replaces the reference's projections (text-decoder.cpp:371-373, 465, 469-472,
// 476-493: GGML mul_mat with GGML_PREC_F32).
//
// Swap-AB: the MMA's M side is 128 weight rows (output features) and its N
// side is a tile of BN tokens, so a decode step's handful of tokens is a
// legal N (32..256) while the weights stream through at full width.
//
// Persistent: a grid of at most one CTA per SM walks the work units (weight
// tile, token tile, K split) round-robin.  The TMA ring runs on across unit
// boundaries, and the accumulator is double-buffered in TMEM (2 x BN columns)
// so the epilogue of one unit overlaps the MMAs of the next.  Skinny shapes
// split K over units and add with f32 red.add into a zeroed C; unsplit units
// store (or read-add-write for accumulate), which keeps them deterministic.
// The host picks BN and the split count with a small cost model.
//
// CTA = 8 warps: warp 0 TMA producer of the weight tiles, warp 6 TMA producer
// of the token tiles (a warp issues TMA copies at a bounded rate, so two
// issuing warps double the ingest of one CTA), warp 7 prefetches weight tiles
// into L2 a bounded distance ahead of warp 0 (so its loads are L2 hits and the
// ring's refill latency shrinks), warp 1 TMEM allocator + MMA issuer (one
// thread), warps 2..5 epilogue (TMEM lane quadrant = warp % 4, one weight row
// per thread).  Every wait is bounded.
#include "kernels.h"

#include <cuda.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

namespace qkv {

namespace {

constexpr int kBK = 64;                           // K per stage: one 128-byte swizzle atom of bf16
// FP8 (e4m3 x e4m3, kind::f8f6f4): a stage holds the same 128-byte rows, i.e.
// 128 elements of K, and each of its 4 MMAs takes K = 32 (32 bytes, as bf16's 16).
template <bool F8> constexpr int kBKe = F8 ? 128 : 64;
constexpr int kBM = 128;                          // weight rows per tile (MMA M)
constexpr uint32_t kABytes = kBM * kBK * 2;       // 16 KB
constexpr int kGemmThreads = 256;
constexpr int kProducerB = 6;                     // warp that loads the token tiles
constexpr int kPrefetchW = 7;                     // warp that prefetches weight tiles into L2

template <int BN> struct TcTraits {
    static constexpr uint32_t kBBytes = BN * kBK * 2;
    static constexpr int NS = BN <= 32 ? 8 : BN <= 64 ? 8 : BN <= 128 ? 6 : 4;
    static constexpr uint32_t kStage = kABytes + kBBytes;
    static constexpr int kCols = 2 * BN;             // two accumulators (power of two, 64..512 columns)
    static constexpr size_t kSmem = 1024 /*align slack*/ + static_cast<size_t>(NS) * kStage + 256;
};

struct TcParams {
    int M, N, K;
    int ktiles_per_split;
    int tiles_n, tiles_m, splits;   // units = tiles_n * tiles_m * splits
    int w_fastest;                  // unit order: 1 weight tile fastest, 0 token tile fastest
    float *C;
    int accumulate;   // 0: store (one split) / red.add into a zeroed C; 1: add into C
    // Fused SwiGLU (act != nullptr, one split): W holds gate and up rows
    // interleaved one by one (row 2f = gate feature f, row 2f + 1 = up
    // feature f), so a feature's two accumulator rows sit in adjacent TMEM
    // lanes of one epilogue warp; act[M][N/2] (bf16) = silu(gate) * up, C is
    // unused.
    __nv_bfloat16 *act;
    DevError *err;
    // FP8 operands: value of W[n][k] = code x w_scale[n], of X[m][k] = code x
    // x_scale[m]; the epilogue multiplies each accumulator by both.
    const float *w_scale;
    const float *x_scale;
    // Slice mode (> 0, split launches only): split s stores its partial sums
    // into C + s x slice_stride instead of adding them into C, so C needs no
    // zeroing, no atomics run, and the reader sums the slices in order.
    size_t slice_stride;
    // Stream-K (sk_ws non-null, one split): CTA c of G takes iterations
    // [c I / G, (c + 1) I / G) of the launch's I = tiles x k-tiles (tiles in
    // the unit order), cut into one segment per tile it touches.  The segment
    // holding a tile's k-tile 0 finishes the tile: it adds, in k order, the
    // partial sums the tile's other segments (the first segments of the next
    // CTAs) left in sk_ws[tile][part][128 rows][BN] and runs the epilogue.
    // sk_flags[tile][4] count the parts each epilogue warp's 32 rows have
    // received; the finishing warp resets its count.
    float *sk_ws;
    int *sk_flags;
};

constexpr int kSkMaxParts = 4;     // stream-K: partial segments a tile may have

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// K-major operand tile of R rows x 64 bf16 with the 128-byte swizzle: rows are
// 128 B, 8-row groups 1024 B apart (SBO), LBO unused (1), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void *tile) {
    const uint64_t addr = smem_u32(tile);
    uint64_t d = 0;
    d |= (addr >> 4) & 0x3FFFull;          // start address
    d |= 1ull << 16;                       // leading byte offset (ignored for swizzled K-major)
    d |= (1024ull >> 4) << 32;             // stride byte offset
    d |= 1ull << 46;                       // descriptor version (sm_100)
    d |= 2ull << 61;                       // SWIZZLE_128B
    return d;
}

// Instruction descriptor, both operands K-major, f32 accumulator, M = 128,
// N = BN: bf16 x bf16 (kind::f16, A and B format 1) or e4m3 x e4m3
// (kind::f8f6f4, A and B format 0).
template <int BN, bool F8> __device__ __forceinline__ uint32_t idesc_mma() {
    const uint32_t ab = F8 ? 0u : ((1u << 7) | (1u << 10));
    return (1u << 4) | ab | (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(kBM >> 4) << 24);
}

template <bool F8>
__device__ __forceinline__ void mma_issue(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, int accum) {
    if constexpr (F8) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(da), "l"(db), "r"(idesc), "r"(accum)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(da), "l"(db), "r"(idesc), "r"(accum)
            : "memory");
    }
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 consecutive TMEM columns of this warp's 32 lanes; the caller waits (tcgen05.wait::ld).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ bool bounded_wait(uint64_t *bar, uint32_t parity) {
    return mbar_wait(bar, parity, kWaitLimitCycles);
}

template <int BN, bool F8>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, TcParams p) {
    using T = TcTraits<BN>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled tiles.
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *tiles = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(tiles + static_cast<size_t>(T::NS) * T::kStage);
    uint64_t *empty = full + T::NS;
    uint64_t *acc_full = empty + T::NS;      // [2] MMA -> epilogue
    uint64_t *acc_empty = acc_full + 2;      // [2] epilogue -> MMA
    uint64_t *mma_done = acc_empty + 2;      // MMA thread's own drain
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
    volatile int *failed = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int *w_issued = failed + 1;     // weight tiles warp 0 has issued (prefetch distance)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ktiles = p.K / kBKe<F8>;
    const int units = p.tiles_n * p.tiles_m * p.splits;
    // The next kernel may start its own set-up now.  Weight tiles depend on no
    // earlier kernel, so their producer starts before pdl_wait; the token-tile
    // producer and the epilogue wait for the previous kernel first.
    pdl_trigger();

    if (threadIdx.x == 0) {
        for (int s = 0; s < T::NS; ++s) {
            mbar_init(&full[s], 2);         // one arrive.expect_tx per producer warp
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(mma_done, 1);
        *failed = 0;
        *w_issued = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(T::kCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Work items of this CTA, in order: round-robin units (tile, K split), or
    // with stream-K one segment per tile of the CTA's iteration range.
    const int n_tiles = p.tiles_m * p.tiles_n;
    const bool sk = p.sk_ws != nullptr;
    const int64_t sk_iters = static_cast<int64_t>(n_tiles) * ktiles;
    const int64_t sk_beg = sk ? static_cast<int64_t>(blockIdx.x) * sk_iters / gridDim.x : 0;
    const int64_t sk_end = sk ? static_cast<int64_t>(blockIdx.x + 1) * sk_iters / gridDim.x : 0;
    auto tile_coords = [&](int t, int &n0, int &m0) {
        const int tm = p.w_fastest ? t / p.tiles_n : t % p.tiles_m;
        const int tn = p.w_fastest ? t % p.tiles_n : t / p.tiles_m;
        n0 = tn * kBM;
        m0 = tm * BN;
    };
    auto first_item = [&]() -> int64_t { return sk ? sk_beg : static_cast<int64_t>(blockIdx.x); };
    auto next_item = [&](int64_t &cur, int &n0, int &m0, int &kt0, int &nk, int &tile) -> bool {
        if (sk) {
            if (cur >= sk_end) return false;
            tile = static_cast<int>(cur / ktiles);
            kt0 = static_cast<int>(cur - static_cast<int64_t>(tile) * ktiles);
            const int64_t tile_end = static_cast<int64_t>(tile + 1) * ktiles;
            const int64_t stop = sk_end < tile_end ? sk_end : tile_end;
            nk = static_cast<int>(stop - cur);
            tile_coords(tile, n0, m0);
            cur = stop;
            return true;
        }
        if (cur >= units) return false;
        const int u = static_cast<int>(cur);
        const int sp = u / n_tiles;
        tile = u - sp * n_tiles;
        tile_coords(tile, n0, m0);
        kt0 = sp * p.ktiles_per_split;
        const int kt1 = min(ktiles, kt0 + p.ktiles_per_split);
        nk = kt1 > kt0 ? kt1 - kt0 : 0;
        cur += gridDim.x;
        return true;
    };

    if (warp == 0 || warp == kProducerB) {
        if (lane == 0) {
            const bool is_w = warp == 0;
            if (!is_w) pdl_wait();
            // The operand that every wave of units re-reads stays in L2 (evict_last): the
            // token tiles when they run fastest, the weights when they do.
            const bool keep = is_w == (p.w_fastest != 0);
            const uint64_t pol = keep ? l2_evict_last_policy() : l2_evict_first_policy();
            const CUtensorMap *map = is_w ? &tmW : &tmX;
            const uint32_t bytes = is_w ? kABytes : T::kBBytes;
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
            int it = 0;
            bool bad = false;
            int64_t cur = first_item();
            int n0, m0, kt0, nk, tile;
            while (!bad && next_item(cur, n0, m0, kt0, nk, tile)) {
                for (int i = 0; i < nk; ++i) {
                    const int s = it % T::NS;
                    const uint32_t ph = static_cast<uint32_t>(it / T::NS) & 1u;
                    if (*failed || !bounded_wait(&empty[s], ph ^ 1u)) {
                        report_error(p.err, kErrWaitTimeout, kWhereGemm, blockIdx.x, it);
                        *failed = 1;
                        bad = true;
                        break;
                    }
                    uint8_t *dst = tiles + static_cast<size_t>(s) * T::kStage + (is_w ? 0u : kABytes);
                    mbar_arrive_expect_tx(&full[s], bytes);
                    tma_load_2d(dst, map, (kt0 + i) * kBKe<F8>, is_w ? n0 : m0, &full[s], pol);
                    ++it;
                    if (is_w) *w_issued = it;
                }
            }
            // Drain: every tile this thread asked for has landed before the CTA can exit.
            for (int i = it > T::NS ? it - T::NS : 0; i < it; ++i) {
                if (!bounded_wait(&full[i % T::NS], static_cast<uint32_t>(i / T::NS) & 1u)) {
                    report_error(p.err, kErrWaitTimeout, kWhereGemm, blockIdx.x, -(1 << 21));
                    break;
                }
            }
        }
    } else if (warp == kPrefetchW) {
        if (lane == 0) {
            // Weight tiles into L2, at most kAhead tiles ahead of the weight producer.
            constexpr int kAhead = 2 * T::NS;
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
            int pit = 0;
            bool stop = false;
            int64_t cur = first_item();
            int n0, m0, kt0, nk, tile;
            while (!stop && next_item(cur, n0, m0, kt0, nk, tile)) {
                for (int i = 0; i < nk; ++i, ++pit) {
                    if (pit >= kAhead) {
                        const long long t0 = clock64();
                        while (pit - *w_issued >= kAhead) {
                            if (*failed || clock64() - t0 > kWaitLimitCycles) {
                                stop = true;
                                break;
                            }
                        }
                        if (stop) break;
                    }
                    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                                     reinterpret_cast<uint64_t>(&tmW)),
                                 "r"((kt0 + i) * kBKe<F8>), "r"(n0)
                                 : "memory");
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_mma<BN, F8>();
            int it = 0, j = 0;
            bool bad = false, any = false;
            int64_t cur = first_item();
            int n0, m0, kt0, nk, tile;
            for (; !bad && next_item(cur, n0, m0, kt0, nk, tile); ++j) {
                const int b = j & 1;
                if (*failed || !bounded_wait(&acc_empty[b], (static_cast<uint32_t>(j >> 1) & 1u) ^ 1u)) {
                    report_error(p.err, kErrWaitTimeout, kWhereGemm, blockIdx.x, -(1 << 22) - j);
                    *failed = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + static_cast<uint32_t>(b * BN);
                for (int i = 0; i < nk; ++i) {
                    const int s = it % T::NS;
                    const uint32_t ph = static_cast<uint32_t>(it / T::NS) & 1u;
                    if (*failed || !bounded_wait(&full[s], ph)) {
                        report_error(p.err, kErrWaitTimeout, kWhereGemm, blockIdx.x, -1 - it);
                        *failed = 1;
                        bad = true;
                        break;
                    }
                    tc_fence_after();
                    const uint8_t *a = tiles + static_cast<size_t>(s) * T::kStage;
                    const uint8_t *bb = a + kABytes;
                    const uint64_t da = smem_desc_sw128(a), db = smem_desc_sw128(bb);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        // advance 32 bytes (16 bf16 or 32 e4m3) inside the swizzle atom
                        // (descriptor units of 16 B)
                        mma_issue<F8>(d, da + 2ull * kk, db + 2ull * kk, idesc, (i > 0 || kk > 0) ? 1 : 0);
                    }
                    mma_commit(&empty[s]);
                    any = true;
                    ++it;
                }
                if (bad) break;
                mma_commit(&acc_full[b]);
            }
            // Every MMA this thread issued has completed before TMEM can be freed.
            if (any) {
                mma_commit(mma_done);
                if (!bounded_wait(mma_done, 0)) report_error(p.err, kErrWaitTimeout, kWhereGemm, blockIdx.x, -(1 << 23));
            }
        }
        __syncwarp();
    } else {
        // epilogue: warps 2..5, TMEM lanes 32*(warp%4) .. +31 = weight rows of the unit
        pdl_wait();
        const int q = warp & 3;
        int j = 0;
        int64_t cur = first_item();
        int n0, m0, kt0, nk, tile;
        for (; next_item(cur, n0, m0, kt0, nk, tile); ++j) {
            const int b = j & 1;
            const bool have = bounded_wait(&acc_full[b], static_cast<uint32_t>(j >> 1) & 1u);
            tc_fence_after();
            // Warp-uniform: tcgen05.ld is .sync.aligned, every lane of the warp must issue it.
            if (!__all_sync(0xffffffffu, have && !*failed)) {
                if (lane == 0) {
                    report_error(p.err, kErrWaitTimeout, kWhereGemm, blockIdx.x, (1 << 20) + j);
                    *failed = 1;
                }
                break;
            }
            const int n = n0 + 32 * q + lane;
            const bool split = p.splits > 1;
            const bool fused = p.act != nullptr;
            // Stream-K: a segment without k-tile 0 is part sk_part of its tile and
            // leaves its sums in the workspace; the one with k-tile 0 adds the
            // tile's sk_nparts parts (once they are all in) before its epilogue.
            int sk_part = -1, sk_nparts = 0;
            if (sk) {
                auto cta_of = [&](int64_t pos) {
                    return ((pos + 1) * static_cast<int64_t>(gridDim.x) + sk_iters - 1) / sk_iters - 1;
                };
                const int64_t it0 = static_cast<int64_t>(tile) * ktiles;
                const int64_t c_head = cta_of(it0);
                if (kt0 == 0) sk_nparts = static_cast<int>(cta_of(it0 + ktiles - 1) - c_head);
                else sk_part = static_cast<int>(blockIdx.x - c_head - 1);
                if (sk_nparts > 0) {
                    int ok = 1;
                    if (lane == 0) {
                        volatile int *f = p.sk_flags + tile * 4 + q;
                        const long long t0 = clock64();
                        while (*f < sk_nparts) {
                            if (*failed || clock64() - t0 > kWaitLimitCycles) {
                                ok = 0;
                                break;
                            }
                        }
                    }
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) {
                        if (lane == 0) {
                            report_error(p.err, kErrWaitTimeout, kWhereGemm, blockIdx.x, -(1 << 26) - tile);
                            *failed = 1;
                        }
                        // hand the accumulator back so the MMA thread does not wait on it
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[b]);
                        break;
                    }
                    __threadfence();
                }
            }
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                uint32_t r[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(b * BN + c), r);
                tmem_wait_ld();
                if (c + 32 >= BN) {
                    // accumulator b fully read: hand it back to the MMA thread
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[b]);
                }
                if constexpr (F8) {
                    // dequantise: weight row n's scale times each token's scale
                    const float ws = n < p.N ? __ldg(p.w_scale + n) : 0.0f;
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) {
                        const int m = m0 + c + jj;
                        const float xs = m < p.M ? p.x_scale[m] : 0.0f;
                        r[jj] = __float_as_uint(__uint_as_float(r[jj]) * ws * xs);
                    }
                }
                if (sk_part >= 0) {
                    // a later piece of its tile: the partial sums go to the workspace only
                    float *wsp = p.sk_ws + ((static_cast<size_t>(tile) * kSkMaxParts + sk_part) * kBM + 32 * q + lane) * BN + c;
#pragma unroll
                    for (int jj = 0; jj < 32; jj += 4)
                        __stcg(reinterpret_cast<float4 *>(wsp + jj),
                               make_float4(__uint_as_float(r[jj]), __uint_as_float(r[jj + 1]), __uint_as_float(r[jj + 2]),
                                           __uint_as_float(r[jj + 3])));
                    continue;
                }
                for (int part = 0; part < sk_nparts; ++part) {
                    // the tile's later pieces, added in k order
                    const float *wsp = p.sk_ws + ((static_cast<size_t>(tile) * kSkMaxParts + part) * kBM + 32 * q + lane) * BN + c;
#pragma unroll
                    for (int jj = 0; jj < 32; jj += 4) {
                        const float4 a = __ldcg(reinterpret_cast<const float4 *>(wsp + jj));
                        r[jj] = __float_as_uint(__uint_as_float(r[jj]) + a.x);
                        r[jj + 1] = __float_as_uint(__uint_as_float(r[jj + 1]) + a.y);
                        r[jj + 2] = __float_as_uint(__uint_as_float(r[jj + 2]) + a.z);
                        r[jj + 3] = __float_as_uint(__uint_as_float(r[jj + 3]) + a.w);
                    }
                }
                if (fused) {
                    // Lane pairs (2i, 2i + 1) hold gate and up of feature n / 2 for the
                    // chunk's 32 tokens.  The even lane finishes tokens 0..15, the odd
                    // lane tokens 16..31: each passes its partner the half it does not
                    // finish (register indices stay compile-time on both sides).
                    const bool gate = (lane & 1) == 0;
                    const int F = p.N >> 1;
                    const int f = n >> 1;
                    const int t0 = gate ? 0 : 16;
                    const int mlim = p.M - (m0 + c);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const float mine = __uint_as_float(gate ? r[jj] : r[16 + jj]);
                        const float other = __shfl_xor_sync(0xffffffffu, __uint_as_float(gate ? r[16 + jj] : r[jj]), 1);
                        const float g = gate ? mine : other, u = gate ? other : mine;
                        if (t0 + jj < mlim && f < F) {
                            // the SwiGLU kernel's formula (accurate exp, IEEE divide)
                            const float sl = g / (1.0f + expf(-g));
                            p.act[static_cast<size_t>(m0 + c + t0 + jj) * F + f] = __float2bfloat16_rn(sl * u);
                        }
                    }
                    continue;
                }
                if (n < p.N) {
                    float *dst = p.C + static_cast<size_t>(m0 + c) * p.N + n;
                    const bool to_slice = split && p.slice_stride > 0;
                    if (to_slice) dst += static_cast<size_t>(kt0 / p.ktiles_per_split) * p.slice_stride;
                    const int mlim = p.M - (m0 + c);
                    if (!split && p.accumulate) {
                        // Read the chunk's 32 C values first (one memory latency, not 32:
                        // the compiler cannot tell that the strided addresses differ).
                        float old[32];
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj)
                            old[jj] = jj < mlim ? dst[static_cast<size_t>(jj) * p.N] : 0.0f;
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj)
                            if (jj < mlim) dst[static_cast<size_t>(jj) * p.N] = old[jj] + __uint_as_float(r[jj]);
                    } else {
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) {
                            if (jj < mlim) {
                                const float v = __uint_as_float(r[jj]);
                                float *dp = dst + static_cast<size_t>(jj) * p.N;
                                if (split && !to_slice) atomicAdd(dp, v);
                                else *dp = v;
                            }
                        }
                    }
                }
            }
            if (sk_part >= 0) {
                // this warp's 32 rows of the part are in: count them for the finishing CTA
                __threadfence();
                __syncwarp();
                if (lane == 0) atomicAdd(p.sk_flags + tile * 4 + q, 1);
            } else if (sk_nparts > 0 && lane == 0) {
                p.sk_flags[tile * 4 + q] = 0;   // every part arrived and was added: ready for the next launch
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(T::kCols) : "memory");
    }
}

// ---- host: tensor maps through the driver entry point (no -lcuda) ----

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

// Matrix [rows][K] (row-major) of bf16 (es = 2) or one-byte codes (es = 1),
// box = box_rows x one 128-byte row segment (64 bf16 / 128 codes), 128-byte swizzle.
bool make_map(CUtensorMap *m, const void *ptr, int rows, int K, int box_rows, int es) {
    EncodeTiled enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * es};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / es), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, es == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
               const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct MapKey {
    const void *ptr;
    int rows, K, box, es;
    bool operator==(const MapKey &o) const {
        return ptr == o.ptr && rows == o.rows && K == o.K && box == o.box && es == o.es;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey &k) const {
        return std::hash<const void *>()(k.ptr) ^ (static_cast<size_t>(k.rows) * 1000003u) ^
               (static_cast<size_t>(k.K) << 20) ^ static_cast<size_t>(k.box) ^ (static_cast<size_t>(k.es) << 40);
    }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

bool cached_map(CUtensorMap *out, const void *ptr, int rows, int K, int box, int es = 2) {
    std::lock_guard<std::mutex> lock(g_map_mu);
    const MapKey key{ptr, rows, K, box, es};
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
        *out = it->second;
        return true;
    }
    if (g_maps.size() > 4096) g_maps.clear();
    CUtensorMap m;
    if (!make_map(&m, ptr, rows, K, box, es)) return false;
    g_maps.emplace(key, m);
    *out = m;
    return true;
}

template <int BN> cudaError_t prepare_bn() {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(TcTraits<BN>::kSmem));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(gemm_tc_kernel<BN, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(TcTraits<BN>::kSmem));
}

// Zeroes C before a K-split GEMM adds its partial sums into it.  A kernel
// rather than a memset, so the launch chain (programmatic dependent launch)
// is not broken: the GEMM behind it starts and streams its weights while this
// and the kernels before it finish.
__global__ void zero_f32_kernel(float4 *c, size_t n4) {
    pdl_trigger();
    pdl_wait();   // earlier kernels may still read C
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        c[i] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// Unit order: weight tiles fastest once the token operand outgrows a share of
// L2 (the weights, <= 50 MB for every decoder projection, then stay resident
// while the token tiles stream once); token tiles fastest otherwise.
bool weight_fastest(int M, int K, int tiles_m) {
    static const char *forced = getenv("QWENASR_B200_GEMM_ORDER");
    if (forced && (forced[0] == 'w' || forced[0] == 't')) return forced[0] == 'w' && tiles_m > 1;
    return tiles_m > 1 && static_cast<double>(M) * K * 2.0 > 32.0e6;
}

template <int BN, bool F8 = false>
cudaError_t launch_bn(const void *X, const void *W, float *C, int M, int N, int K, int accumulate, int splits,
                      int num_sms, DevError *err, cudaStream_t st, __nv_bfloat16 *act = nullptr,
                      const float *w_scale = nullptr, const float *x_scale = nullptr, bool slices = false,
                      float *sk_ws = nullptr, int *sk_flags = nullptr) {
    CUtensorMap tw, tx;
    const int es = F8 ? 1 : 2;
    if (!cached_map(&tw, W, N, K, kBM, es) || !cached_map(&tx, X, M, K, BN, es)) return cudaErrorInvalidValue;
    const int tiles_n = (N + kBM - 1) / kBM, tiles_m = (M + BN - 1) / BN;
    const int ktiles = K / kBKe<F8>;
    const int kps = (ktiles + splits - 1) / splits;
    splits = (ktiles + kps - 1) / kps;     // every split owns >= 1 k-tile
    if (act && splits != 1) return cudaErrorInvalidValue;
    if (slices && accumulate) return cudaErrorInvalidValue;
    if (splits > 1 && !accumulate && !slices) {
        const size_t n = static_cast<size_t>(M) * N;
        cudaError_t e;
        if (n % 4 == 0 && (reinterpret_cast<uintptr_t>(C) & 15) == 0) {
            const size_t blocks = (n / 4 + 255) / 256;
            e = launch_pdl(zero_f32_kernel, dim3(static_cast<unsigned>(blocks < 1184 ? blocks : 1184)), dim3(256), 0,
                           st, reinterpret_cast<float4 *>(C), n / 4);
        } else {
            e = cudaMemsetAsync(C, 0, n * sizeof(float), st);
        }
        if (e != cudaSuccess) return e;
    }
    if (sk_ws && (splits != 1 || !sk_flags)) return cudaErrorInvalidValue;
    TcParams p{M, N, K, kps, tiles_n, tiles_m, splits, weight_fastest(M, K * es / 2, tiles_m) ? 1 : 0, C, accumulate,
               act, err, w_scale, x_scale, slices && splits > 1 ? static_cast<size_t>(M) * N : size_t{0}, sk_ws,
               sk_flags};
    const int units = tiles_n * tiles_m * splits;
    const int grid = sk_ws ? num_sms : (units < num_sms ? units : num_sms);
    return launch_pdl(gemm_tc_kernel<BN, F8>, dim3(grid), dim3(kGemmThreads), TcTraits<BN>::kSmem, st, tw, tx, p);
}

// Cost model for the tile width BN and the K split.  One thread issues a
// tcgen05.mma (M=128, K=16) about every 150 cycles whatever N is, so a
// k-tile (4 MMAs) costs about the same for every BN and only N = 256 keeps
// the tensor pipe busy; below that a k-tile is bounded by MMA issue, by the
// operand bytes the two TMA warps bring in, and by the refill latency over
// the ring depth.  Units run round-robin over the persistent CTAs; a split
// adds red.add traffic into C (and a memset when not accumulating).
struct GemmPlan {
    int bn, splits;
};

template <int BN> constexpr double ktile_seconds() {
    constexpr double kClk = 1.9e9;
    constexpr double t_mma = 4 * 150.0 / kClk;                                    // issue-bound MMAs
    constexpr double t_ld = (kABytes + TcTraits<BN>::kBBytes) / 150e9;           // two TMA issuers
    constexpr double t_lat = 1.3e-6 / (TcTraits<BN>::NS - 1);                     // refill latency / depth
    return t_mma > t_ld ? (t_mma > t_lat ? t_mma : t_lat) : (t_ld > t_lat ? t_ld : t_lat);
}

// slices: the launch stores each split's partial sums into its own slice
// (plain stores, summed by the reader) instead of adding them into C with
// red.add after a zeroing kernel.
GemmPlan plan_gemm(int M, int N, int K, int num_sms, bool no_split = false, bool f8 = false, bool slices = false) {
    const double kHbm = 6.2e12;                     // whole-chip weight streaming
    const double kFixed = 1.5e-6;                   // per-unit fill + epilogue tail
    const double kRed = 250e9;                      // f32 red.add per second, whole chip
    const int ktiles = K / (f8 ? kBKe<true> : kBK);   // a k-tile is 128 bytes of K either way
    const int tiles_n = (N + kBM - 1) / kBM;
    const double tk[4] = {ktile_seconds<32>(), ktile_seconds<64>(), ktile_seconds<128>(), ktile_seconds<256>()};
    GemmPlan best{256, 1};
    double best_t = 1e30;
    int bi = 0;
    for (int bn : {32, 64, 128, 256}) {
        const int idx = bi++;
        if (bn > 32 && (bn / 2) >= M) break;          // a narrower tile already covers all tokens
        const int tiles_m = (M + bn - 1) / bn;
        const int tiles = tiles_n * tiles_m;
        const int max_split = no_split ? 1 : (ktiles < 32 ? ktiles : 32);
        for (int sp = 1; sp <= max_split; ++sp) {
            const int kps = (ktiles + sp - 1) / sp;
            const int spr = (ktiles + kps - 1) / kps;
            if (spr != sp) continue;
            const long units = static_cast<long>(tiles) * sp;
            const long waves = (units + num_sms - 1) / num_sms;
            double t = waves * (kps * tk[idx] + kFixed);
            const double t_w = static_cast<double>(N) * K * (f8 ? 1.0 : 2.0) / kHbm;   // weights read from HBM once
            if (t_w > t) t = t_w;
            if (sp > 1) {
                if (slices) t += static_cast<double>(M) * N * sp * 4.0 / 3.0e12;   // slice stores (read back from L2)
                else t += static_cast<double>(M) * N * sp / kRed + 1.0e-6;         // red.add + the zeroing kernel
            }
            if (t < best_t * 0.98) {
                best_t = t;
                best = {bn, sp};
            }
        }
    }
    return best;
}

}  // namespace

bool tc_tensor_map(CUtensorMap *out, const void *ptr, int rows, int K, int box_rows) {
    return cached_map(out, ptr, rows, K, box_rows);
}

cudaError_t prepare_gemm_tc() {
    cudaError_t e;
    if ((e = prepare_bn<32>()) != cudaSuccess) return e;
    if ((e = prepare_bn<64>()) != cudaSuccess) return e;
    if ((e = prepare_bn<128>()) != cudaSuccess) return e;
    return prepare_bn<256>();
}

bool gemm_tc_supported(int M, int N, int K) {
    return M > 0 && N > 0 && K > 0 && K % kBK == 0 && encoder() != nullptr;
}

namespace {
GemmPlan choose_plan(int M, int N, int K, int num_sms) {
    GemmPlan pl = plan_gemm(M, N, K, num_sms);
    // Tuning override: QWENASR_B200_GEMM_PLAN="bn,splits" forces the plan (sweeps).
    static const char *forced = getenv("QWENASR_B200_GEMM_PLAN");
    if (forced) {
        int bn = 0, sp = 0;
        if (sscanf(forced, "%d,%d", &bn, &sp) == 2 && (bn == 32 || bn == 64 || bn == 128 || bn == 256) && sp >= 1)
            pl = {bn, sp};
    }
    return pl;
}
}  // namespace

int gemm_tc_kernels(int M, int N, int K, int accumulate, int num_sms) {
    if (M <= 0 || N <= 0 || K % kBK != 0) return 0;
    const GemmPlan pl = choose_plan(M, N, K, num_sms);
    const int ktiles = K / kBK;
    const int kps = (ktiles + pl.splits - 1) / pl.splits;
    const int splits = (ktiles + kps - 1) / kps;
    return (splits > 1 && !accumulate) ? 2 : 1;
}

cudaError_t launch_gemm_tc(const void *X, const void *W, float *C, int M, int N, int K, int accumulate, int num_sms,
                           DevError *err, cudaStream_t st) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (K % kBK != 0) return cudaErrorInvalidValue;
    const GemmPlan pl = choose_plan(M, N, K, num_sms);
    switch (pl.bn) {
        case 32: return launch_bn<32>(X, W, C, M, N, K, accumulate, pl.splits, num_sms, err, st);
        case 64: return launch_bn<64>(X, W, C, M, N, K, accumulate, pl.splits, num_sms, err, st);
        case 128: return launch_bn<128>(X, W, C, M, N, K, accumulate, pl.splits, num_sms, err, st);
        default: return launch_bn<256>(X, W, C, M, N, K, accumulate, pl.splits, num_sms, err, st);
    }
}

bool gemm_tc_fp8_supported(int M, int N, int K) {
    return M > 0 && N > 0 && K > 0 && K % kBKe<true> == 0 && encoder() != nullptr;
}

int gemm_tc_fp8_kernels(int M, int N, int K, int accumulate, int num_sms) {
    if (!gemm_tc_fp8_supported(M, N, K)) return 0;
    const GemmPlan pl = plan_gemm(M, N, K, num_sms, false, true);
    const int ktiles = K / kBKe<true>;
    const int kps = (ktiles + pl.splits - 1) / pl.splits;
    const int splits = (ktiles + kps - 1) / kps;
    return (splits > 1 && !accumulate) ? 2 : 1;
}

cudaError_t launch_gemm_tc_fp8(const void *X, const float *x_scale, const void *W, const float *w_scale, float *C,
                               int M, int N, int K, int accumulate, int num_sms, DevError *err, cudaStream_t st) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (!gemm_tc_fp8_supported(M, N, K) || !x_scale || !w_scale) return cudaErrorInvalidValue;
    const GemmPlan pl = plan_gemm(M, N, K, num_sms, false, true);
    switch (pl.bn) {
        case 32: return launch_bn<32, true>(X, W, C, M, N, K, accumulate, pl.splits, num_sms, err, st, nullptr, w_scale, x_scale);
        case 64: return launch_bn<64, true>(X, W, C, M, N, K, accumulate, pl.splits, num_sms, err, st, nullptr, w_scale, x_scale);
        case 128: return launch_bn<128, true>(X, W, C, M, N, K, accumulate, pl.splits, num_sms, err, st, nullptr, w_scale, x_scale);
        default: return launch_bn<256, true>(X, W, C, M, N, K, accumulate, pl.splits, num_sms, err, st, nullptr, w_scale, x_scale);
    }
}

namespace {
template <bool F8>
cudaError_t launch_slices(const void *X, const float *x_scale, const void *W, const float *w_scale, float *C, int M,
                          int N, int K, int max_slices, int num_sms, DevError *err, cudaStream_t st, int *slices) {
    if (M <= 0 || N <= 0) {
        *slices = 1;
        return cudaSuccess;
    }
    if (K % kBKe<F8> != 0 || max_slices < 1) return cudaErrorInvalidValue;
    const GemmPlan pl = plan_gemm(M, N, K, num_sms, false, F8, true);
    const int ktiles = K / kBKe<F8>;
    const int want = pl.splits < max_slices ? pl.splits : max_slices;
    const int kps = (ktiles + want - 1) / want;
    *slices = (ktiles + kps - 1) / kps;
    switch (pl.bn) {
        case 32: return launch_bn<32, F8>(X, W, C, M, N, K, 0, want, num_sms, err, st, nullptr, w_scale, x_scale, true);
        case 64: return launch_bn<64, F8>(X, W, C, M, N, K, 0, want, num_sms, err, st, nullptr, w_scale, x_scale, true);
        case 128: return launch_bn<128, F8>(X, W, C, M, N, K, 0, want, num_sms, err, st, nullptr, w_scale, x_scale, true);
        default: return launch_bn<256, F8>(X, W, C, M, N, K, 0, want, num_sms, err, st, nullptr, w_scale, x_scale, true);
    }
}
}  // namespace

cudaError_t launch_gemm_tc_slices(const void *X, const void *W, float *C, int M, int N, int K, int max_slices,
                                  int num_sms, DevError *err, cudaStream_t st, int *slices) {
    return launch_slices<false>(X, nullptr, W, nullptr, C, M, N, K, max_slices, num_sms, err, st, slices);
}

cudaError_t launch_gemm_tc_fp8_slices(const void *X, const float *x_scale, const void *W, const float *w_scale,
                                      float *C, int M, int N, int K, int max_slices, int num_sms, DevError *err,
                                      cudaStream_t st, int *slices) {
    if (!x_scale || !w_scale) return cudaErrorInvalidValue;
    return launch_slices<true>(X, x_scale, W, w_scale, C, M, N, K, max_slices, num_sms, err, st, slices);
}

bool gemm_tc_swiglu_pays(int M, int N2, int K, int num_sms) {
    // The fused GEMM runs unsplit.  It pays where the plain GEMM would not
    // split either (the same GEMM, with the SwiGLU launch and the f32 gate/up
    // round trip gone), and where every CTA takes two or more units anyway.
    if (K % kBK != 0 || N2 % 2 != 0) return false;
    if (plan_gemm(M, N2, K, num_sms).splits == 1) return true;
    const GemmPlan pl = plan_gemm(M, N2, K, num_sms, true);
    const long units = static_cast<long>(N2 / kBM) * ((M + pl.bn - 1) / pl.bn);
    return units >= 2L * num_sms;
}

// Stream-K for a launch of `tiles` output tiles of k-tiles each on `num_sms`
// CTAs: worth it when the tiles leave SMs idle, possible when every tile's
// pieces fit kSkMaxParts and the workspace holds them.
bool stream_k_fits(int tiles, int ktiles, int bn, int num_sms, size_t ws_floats, int flag_tiles) {
    if (tiles >= num_sms || bn > 64 || tiles > flag_tiles) return false;
    if (static_cast<size_t>(tiles) * kSkMaxParts * kBM * bn > ws_floats) return false;
    const int64_t I = static_cast<int64_t>(tiles) * ktiles, G = num_sms;
    if (I < 2 * G) return false;   // under two k-tiles per CTA: too little work to split
    auto cta_of = [&](int64_t pos) { return ((pos + 1) * G + I - 1) / I - 1; };
    for (int t = 0; t < tiles; ++t) {
        const int64_t i0 = static_cast<int64_t>(t) * ktiles;
        if (cta_of(i0 + ktiles - 1) - cta_of(i0) > kSkMaxParts) return false;
    }
    return true;
}

cudaError_t launch_gemm_tc_swiglu(const void *X, const void *W, void *act, int M, int N2, int K, int num_sms,
                                  DevError *err, cudaStream_t st, float *sk_ws, int *sk_flags, size_t sk_ws_floats,
                                  int sk_flag_tiles) {
    if (M <= 0 || N2 <= 0) return cudaSuccess;
    if (K % kBK != 0 || N2 % 2 != 0) return cudaErrorInvalidValue;
    GemmPlan pl = plan_gemm(M, N2, K, num_sms, true);
    const int tiles = ((N2 + kBM - 1) / kBM) * ((M + pl.bn - 1) / pl.bn);
    const bool use_sk = sk_ws && sk_flags && stream_k_fits(tiles, K / kBK, pl.bn, num_sms, sk_ws_floats, sk_flag_tiles);
    float *ws = use_sk ? sk_ws : nullptr;
    int *fl = use_sk ? sk_flags : nullptr;
    __nv_bfloat16 *a = static_cast<__nv_bfloat16 *>(act);
    switch (pl.bn) {
        case 32: return launch_bn<32>(X, W, nullptr, M, N2, K, 0, 1, num_sms, err, st, a, nullptr, nullptr, false, ws, fl);
        case 64: return launch_bn<64>(X, W, nullptr, M, N2, K, 0, 1, num_sms, err, st, a, nullptr, nullptr, false, ws, fl);
        case 128: return launch_bn<128>(X, W, nullptr, M, N2, K, 0, 1, num_sms, err, st, a);
        default: return launch_bn<256>(X, W, nullptr, M, N2, K, 0, 1, num_sms, err, st, a);
    }
}

}  // namespace qkv
