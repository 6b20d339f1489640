// K2: paged GQA decode attention (one query token per row), HBM-bound, no
// tensor cores.  Replaces text-decoder.cpp:435-463 (mul_mat over the full
// cache view, soft_max_ext with a host mask, cont(transpose(V)) copy of all of
// V every step, second mul_mat) and the scalar twin :1029-1075.
//
// Work split ("stream-K over pages"): all rows' pages are laid end to end
// (prefix sums of ceil(len/16)); CTA c of G takes the page range
// [c*T/G, (c+1)*T/G), so every CTA streams the same number of bytes whatever
// the context-length mix.  A range may cover the tail of one row, several
// whole rows and the head of another: each (CTA, row) piece is a segment.  A
// row covered by one CTA writes its output directly; a row split over CTAs
// c0..c1 writes unnormalised partials (O, m, l) to scratch slot row + c (that
// index is unique per segment) and the last of its segments to finish (per kv
// head, atomic counter) merges them.  Counters reset themselves.
//
// CTA = HALVES x 8 consumer warps + 1 producer warp + 3 append warps (busy
// only with the append-ahead of the next layer, AttendParams::next).
// Consumer warp g (and, with HALVES = 2, warp g + 8) serves kv head g (q
// heads 2g and 2g+1).  With
// two halves each warp keeps its own online-softmax state; at the end of a
// segment warp g + 8 hands (m, l, O) to warp g through shared memory (bounded
// flag waits) and warp g merges.  The halves share a head's work in one of two
// ways.  bf16: both warps read every stage and each takes 8 of the page's 16
// tokens, which halves the dependent chain (loads, dots, shuffles, exp2, PV)
// a warp runs per page, so a stage is handed back sooner and more of the ring
// is in flight.  8-bit caches: the warps take alternate chunks of a 6-stage
// ring (a dequant per element on top of the bf16 work needs twice the loads,
// conversions and FMA chains in flight); a stage must then always be consumed
// by the same half (a warp that skipped a phase of a stage's mbarrier could
// otherwise see the parity of the phase before it), so NS is a multiple of
// HALVES.  The producer streams each page chunk (all 8 heads, K and
// V) into an NS-stage shared-memory ring with cp.async.bulk (no tensor map,
// no multicast), completion on mbarriers.  Every wait is bounded.
//
// Consumer math per chunk of CH tokens (bf16/fp8: CH = 16 = one page, f32: 8):
//   QK: lane = (quarter qt, dim group j): tokens qt*WT/4.. of the warp's WT
//       tokens (WT = CH, or CH / 2 when the halves split the tokens), dims = 16 per lane
//       in 16-byte chunks j, j+8, ... (conflict-free smem reads), partial dots
//       reduce-scattered over the 8 lanes of the quarter.
//   softmax: online (running max m, sum l) in the log2 domain (q pre-scaled
//       by log2(e)/sqrt(D)); p exchanged through a per-warp smem row.
//   PV: lane owns dims [4*lane, 4*lane+4) of both heads.
#include "kernels.h"

#include <cmath>
#include <cstring>
#include <mutex>

#include "kappend.cuh"
#include "qkv.h"

namespace qkv {

namespace {

// CH: tokens per ring chunk; NS: ring stages; HALVES: consumer warps per kv
// head; TSPLIT: with two halves, whether they split each chunk's tokens
// (true: both read every stage) or take alternate chunks (false).
template <typename TC> struct AttnTraits;
template <> struct AttnTraits<__nv_bfloat16> {
    static constexpr int CH = 16, NS = 3, HALVES = 2;
    static constexpr bool TSPLIT = true;
};
template <> struct AttnTraits<float> {
    static constexpr int CH = 8, NS = 3, HALVES = 1;
    static constexpr bool TSPLIT = false;
};
template <> struct AttnTraits<uint8_t> {
    static constexpr int CH = 16, NS = 6, HALVES = 2;
    static constexpr bool TSPLIT = false;
};

template <typename TC> __host__ __device__ constexpr int consumers() { return kHkv * AttnTraits<TC>::HALVES; }
// Warps that do the append-ahead (AttendParams::next), idle otherwise: three
// keep the CTA at 5 warps per scheduler with the consumers' register budget
// unchanged.
constexpr int kAppendWarps = 3;
template <typename TC> __host__ __device__ constexpr int threads() {
    return (consumers<TC>() + 1 + kAppendWarps) * 32;
}

template <typename TC> __host__ __device__ constexpr uint32_t stage_bytes() {
    return 2u * kHkv * AttnTraits<TC>::CH * kHeadDim * sizeof(TC);
}
template <typename TC> __host__ __device__ constexpr size_t smem_bytes() {
    return static_cast<size_t>(AttnTraits<TC>::NS) * stage_bytes<TC>()    // stages
           + 2 * AttnTraits<TC>::NS * sizeof(uint64_t)                      // full/empty barriers
           + AttnTraits<TC>::NS * kPageScales * sizeof(float)               // 8-bit scales per stage
           + consumers<TC>() * 2 * AttnTraits<TC>::CH * sizeof(float)       // p exchange (16B aligned)
           + kHkv * 32 * 8 * sizeof(float)                                  // half-warp O hand-over
           + kHkv * 4 * sizeof(float)                                       // half-warp (m, l) hand-over
           + (kAttnMaxRows + 1) * sizeof(int)                               // row page prefix
           + 32 * sizeof(int)                                               // scan scratch + abort flag
           + 2 * kHkv * sizeof(int);                                        // hand-over seq / ack flags
}

// Load 16 bytes of cache elements as floats.
template <typename TC> struct Chunk16;
template <> struct Chunk16<__nv_bfloat16> {
    static constexpr int E = 8;
    static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float (&o)[8]) {
        const uint4 w = *reinterpret_cast<const uint4 *>(p);
        o[0] = bf16lo(w.x); o[1] = bf16hi(w.x); o[2] = bf16lo(w.y); o[3] = bf16hi(w.y);
        o[4] = bf16lo(w.z); o[5] = bf16hi(w.z); o[6] = bf16lo(w.w); o[7] = bf16hi(w.w);
    }
};
template <> struct Chunk16<float> {
    static constexpr int E = 4;
    static __device__ __forceinline__ void load(const float *p, float (&o)[4]) {
        const float4 w = *reinterpret_cast<const float4 *>(p);
        o[0] = w.x; o[1] = w.y; o[2] = w.z; o[3] = w.w;
    }
};
template <> struct Chunk16<uint8_t> {
    static constexpr int E = 16;
    static __device__ __forceinline__ void load(const uint8_t *p, float (&o)[16]) {
        const uint4 w = *reinterpret_cast<const uint4 *>(p);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 a = e4m3x2_to_f2(static_cast<uint16_t>(ws[k] & 0xffffu));
            const float2 b = e4m3x2_to_f2(static_cast<uint16_t>(ws[k] >> 16));
            o[4 * k + 0] = a.x; o[4 * k + 1] = a.y; o[4 * k + 2] = b.x; o[4 * k + 3] = b.y;
        }
    }
};

// Four consecutive cache elements as floats (PV rows).
template <typename TC> __device__ __forceinline__ float4 load4(const TC *p);
template <> __device__ __forceinline__ float4 load4<float>(const float *p) {
    return *reinterpret_cast<const float4 *>(p);
}
template <> __device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16 *p) {
    const uint2 w = *reinterpret_cast<const uint2 *>(p);
    return make_float4(bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y));
}

template <typename TOut> __device__ __forceinline__ void store4(TOut *p, float4 v);
template <> __device__ __forceinline__ void store4<float>(float *p, float4 v) {
    *reinterpret_cast<float4 *>(p) = v;
}
template <> __device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16 *p, float4 v) {
    *reinterpret_cast<uint2 *>(p) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
}

// Reduce-scatter NV values over the 8 lanes of a quarter (offsets 4, 2, 1):
// afterwards v[0] holds the full sum of value index k(j); leftover offsets
// are all-reduced.
template <int NV> __device__ __forceinline__ void reduce_scatter8(float (&v)[NV], int j) {
    int o = 4;
#pragma unroll
    for (int cnt = NV; cnt > 1; cnt >>= 1, o >>= 1) {
        const bool upper = (j & o) != 0;
#pragma unroll
        for (int i = 0; i < cnt / 2; ++i) {
            const float send = upper ? v[i] : v[i + cnt / 2];
            const float keep = upper ? v[i + cnt / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
#pragma unroll
    for (; o >= 1; o >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
}

__device__ __forceinline__ int64_t cta_of_page(int64_t pg, int64_t total, int64_t G) {
    return ((pg + 1) * G + total - 1) / total - 1;
}

// Bounded wait that also gives up when another role raised the abort flag.
__device__ __forceinline__ bool stage_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                           long long limit = kWaitLimitCycles) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > limit) return false;
    }
    return true;
}

// Bounded wait until *flag == want (a shared-memory hand-over between two
// warps of the CTA); false on timeout or when another warp set the abort flag.
__device__ __forceinline__ bool flag_wait(volatile int *flag, int want, volatile int *abort_flag,
                                          long long limit = kWaitLimitCycles) {
    if (*flag == want) return true;
    const long long t0 = clock64();
    while (*flag != want) {
        if (*abort_flag) return false;
        if (clock64() - t0 > limit) return false;
    }
    return true;
}

// Wait probe: runs the bounded waits the kernels use against events that
// never come, with a caller-given short limit, so a test can see a wait run
// out and be reported through the device error word while the context stays
// usable.  Warp 0 waits on an mbarrier that expects one arrival nobody makes
// (K2's stage wait, then the plain mbarrier wait of the GEMM and K3); warp 1
// waits on a shared flag nobody sets (K2's hand-over wait).  Nothing is in
// flight when a wait gives up, so the CTA simply returns.
__global__ void __launch_bounds__(64) wait_probe_kernel(DevError *err, long long limit) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int flag, never;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        flag = 0;
        never = 0;
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (lane != 0) return;
    if (warp == 0) {
        if (!stage_wait(&bar, 0u, &never, limit)) report_error(err, kErrWaitTimeout, kWhereProbe, 0, 0);
        if (!mbar_wait(&bar, 0u, limit)) report_error(err, kErrWaitTimeout, kWhereProbe, 1, 0);
    } else {
        if (!flag_wait(&flag, 1, &never, limit)) report_error(err, kErrWaitTimeout, kWhereProbe, 2, 0);
    }
}

// kVI8 (8-bit cache only): V is int8 (excess-128 bytes) rather than e4m3.
template <typename TC, typename TOut, bool kVI8 = false>
__global__ void __launch_bounds__(threads<TC>(), 1) decode_attn_kernel(AttendParams p) {
    pdl_trigger();
    // With p.early the set-up below (row arrays, page table: host copies that
    // finished before the preceding kernels) and the copies of pages other
    // than a row's last run before the grid dependency wait; the producer waits
    // before a row's last page, the consumers before q and the merge scratch.
    if (!p.early) pdl_wait();
    constexpr int CH = AttnTraits<TC>::CH;
    constexpr int NS = AttnTraits<TC>::NS;
    constexpr int kHalves = AttnTraits<TC>::HALVES;
    constexpr int kConsumers = consumers<TC>();
    constexpr int kThreads = threads<TC>();
    constexpr bool kTSplit = AttnTraits<TC>::TSPLIT;
    static_assert(kTSplit || NS % kHalves == 0, "each stage must be consumed by one half");
    static_assert(!kTSplit || (kHalves == 2 && sizeof(TC) == 2), "token split: bf16, two halves");
    constexpr int CPP = kPageTokens / CH;          // chunks per page
    constexpr int HALF = kHkv * CH * kHeadDim;      // elements of K (or V) in a stage
    constexpr int WT = kTSplit ? CH / kHalves : CH; // tokens of a chunk one warp takes
    constexpr int TPQ = WT / 4;                     // tokens per quarter-warp
    constexpr int NV = 2 * TPQ;                     // partial dots per lane
    constexpr int E = Chunk16<TC>::E;               // elements per 16-byte chunk
    constexpr int NC = 16 / E;                      // chunks per lane per row (16 dims)
    constexpr int KSHIFT = (NV == 8) ? 0 : 1;       // value index k = j >> KSHIFT
    constexpr int HB = (NV == 8) ? 1 : 2;           // lane bit that selects the head
    constexpr bool kFp8 = sizeof(TC) == 1;

    extern __shared__ __align__(128) uint8_t smem[];
    TC *stages = reinterpret_cast<TC *>(smem);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + static_cast<size_t>(NS) * stage_bytes<TC>());
    uint64_t *empty = full + NS;
    float *sscale = reinterpret_cast<float *>(empty + NS);
    float *pbuf = sscale + NS * kPageScales;                               // [kConsumers][2*CH]
    float *xo = pbuf + kConsumers * 2 * CH;                                // [kHkv][32 lanes][8]
    float *xml = xo + kHkv * 32 * 8;                                       // [kHkv][m_a, l_a, m_b, l_b]
    int *row_start = reinterpret_cast<int *>(xml + kHkv * 4);             // [kAttnMaxRows + 1]
    int *scan = row_start + kAttnMaxRows + 1;       // [0..19] warp totals, [24] abort flag
    volatile int *abort_flag = scan + 24;
    volatile int *xseq = scan + 32;                 // [kHkv] segments handed over by warp g + 8
    volatile int *xack = xseq + kHkv;               // [kHkv] segments merged by warp g

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = p.n;

    // ---- row page prefix sums (each thread owns 4 consecutive rows) ----
    int cnt[4];
    int local = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int r = tid * 4 + k;
        int pg = 0;
        if (r < n) {
            const int len = p.lens[r];
            pg = (len + kPageTokens - 1) / kPageTokens;
            if (len < 1 || pg > p.maxp) {
                report_error(p.err, kErrRowBounds, kWhereAttend, r, len);
                pg = 0;
            }
        }
        cnt[k] = pg;
        local += pg;
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) scan[warp] = incl;
    if (tid == 0) {
        *abort_flag = 0;
        for (int k = 0; k < kHkv; ++k) xseq[k] = xack[k] = 0;
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            // one arrival per warp that reads the chunk: both halves with a token
            // split, else the one warp per kv head that took it
            mbar_init(&empty[s], kTSplit ? kConsumers : kHkv);
        }
        fence_mbar_init();
    }
    __syncthreads();
    int warp_off = 0;
    for (int w = 0; w < warp; ++w) warp_off += scan[w];
    int excl = warp_off + incl - local;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int r = tid * 4 + k;
        if (r < n) row_start[r] = excl;
        excl += cnt[k];
    }
    if (tid == kThreads - 1) row_start[n] = warp_off + incl;
    __syncthreads();

    const int64_t T = row_start[n];
    // With fewer pages than CTAs, only the first T CTAs take a (one-page) range:
    // every CTA in [0, G) then owns a non-empty range, which the per-row
    // segment count c1 - c0 + 1 below relies on.
    const int64_t G = T < static_cast<int64_t>(gridDim.x) ? T : static_cast<int64_t>(gridDim.x);
    const int64_t c = blockIdx.x;
    if (c >= G) return;     // no pages for this CTA (nothing armed yet)
    const int64_t pb = c * T / G, pe = (c + 1) * T / G;
    int r0 = 0;
    {
        int lo = 0, hi = n - 1;
        while (lo < hi) {   // largest r with row_start[r] <= pb
            const int mid = (lo + hi + 1) >> 1;
            if (row_start[mid] <= pb) lo = mid; else hi = mid - 1;
        }
        r0 = lo;
    }

    static_assert(kConsumers + 1 + kAppendWarps <= 24, "warp totals must fit below the abort flag");
    if (warp > kConsumers) {
        // ===== append warps: K1's work for the next layer (append-ahead) =====
        // Rows dealt evenly over the G active CTAs, 16 warp tasks per row
        // (two half-warp units each), after the grid dependency wait: the
        // next layer's q buffer was read by the launch before this one.
        const AppendParams &a = p.next;
        if (a.n <= 0) return;
        pdl_wait();
        const int ra = static_cast<int>(c * a.n / G), rb = static_cast<int>((c + 1) * a.n / G);
        const int aw = warp - kConsumers - 1;
#pragma unroll 1
        for (int task = aw; task < (rb - ra) * 16; task += kAppendWarps)
            append_row_unit<TC>(a, ra + task / 16, 2 * (task % 16) + (lane >> 4), lane & 15);
        return;
    }
    if (warp == kConsumers) {
        // ================= producer warp =================
        const uint64_t pol = l2_evict_first_policy();
        const TC *pool = static_cast<const TC *>(p.pool);
        int iter = 0;
        bool abort = false;
        bool waited = !p.early;
        int r = r0;
        int64_t gp = pb;
        while (gp < pe && !abort) {
            while (row_start[r + 1] <= gp) ++r;
            const int rs = row_start[r];
            const int row_pages = row_start[r + 1] - rs;
            const int j0 = static_cast<int>(gp - rs);
            const int j1 = static_cast<int>((pe < row_start[r + 1] ? pe : row_start[r + 1]) - rs);
            const int slot = p.slots[r];
            if (slot < 0 || slot >= p.max_streams) {
                if (lane == 0) report_error(p.err, kErrRowBounds, kWhereAttend, r, slot);
                abort = true;
                break;
            }
            for (int jb = j0; jb < j1 && !abort; jb += 32) {
                const int jj = jb + lane;
                int pid = 0;
                bool bad = false;
                if (jj < j1) {
                    pid = p.page_table[static_cast<size_t>(slot) * p.maxp + jj];
                    bad = pid < 0 || pid >= p.n_pages;
                }
                if (__any_sync(0xffffffffu, bad)) {
                    if (bad) report_error(p.err, kErrPageIndex, kWhereAttend, r, pid);
                    abort = true;
                    break;
                }
                const int cntp = (j1 - jb) < 32 ? (j1 - jb) : 32;
                for (int k = 0; k < cntp && !abort; ++k) {
                    const int page = __shfl_sync(0xffffffffu, pid, k);
                    if (!waited && jb + k == row_pages - 1) {
                        pdl_wait();   // the row's last page holds this step's token
                        waited = true;
                    }
#pragma unroll 1
                    for (int cp = 0; cp < CPP; ++cp) {
                        const int s = iter % NS;
                        const uint32_t ph = static_cast<uint32_t>(iter / NS) & 1u;
                        int ok = 1;
                        if (lane == 0) {
                            if (!stage_wait(&empty[s], ph ^ 1u, abort_flag)) {
                                ok = 0;
                            } else {
                                TC *dst = stages + static_cast<size_t>(s) * (2 * HALF);
                                const size_t kbase = (static_cast<size_t>(page) * 2) * kPageHalfElems;
                                const size_t vbase = kbase + kPageHalfElems;
                                if constexpr (CH == kPageTokens) {
                                    // K and V halves of a page are contiguous: one copy (a CTA
                                    // issues bulk copies at a bounded rate, so bytes per copy count).
                                    constexpr uint32_t half_bytes = HALF * sizeof(TC);
                                    constexpr uint32_t scale_bytes = kFp8 ? kPageScales * sizeof(float) : 0u;
                                    mbar_arrive_expect_tx(&full[s], 2 * half_bytes + scale_bytes);
                                    bulk_g2s(dst, pool + kbase, 2 * half_bytes, &full[s], pol);
                                    if constexpr (kFp8) {
                                        bulk_g2s(sscale + s * kPageScales,
                                                 p.scales + static_cast<size_t>(page) * kPageScales, scale_bytes,
                                                 &full[s], pol);
                                    }
                                } else {
                                    constexpr uint32_t rows_bytes = CH * kHeadDim * sizeof(TC);
                                    mbar_arrive_expect_tx(&full[s], 2 * kHkv * rows_bytes);
#pragma unroll 1
                                    for (int g = 0; g < kHkv; ++g) {
                                        const size_t off = static_cast<size_t>(g) * kPageTokens * kHeadDim +
                                                           static_cast<size_t>(cp) * CH * kHeadDim;
                                        bulk_g2s(dst + g * CH * kHeadDim, pool + kbase + off, rows_bytes, &full[s], pol);
                                        bulk_g2s(dst + HALF + g * CH * kHeadDim, pool + vbase + off, rows_bytes, &full[s], pol);
                                    }
                                }
                            }
                        }
                        ok = __shfl_sync(0xffffffffu, ok, 0);
                        if (!ok) {
                            if (lane == 0) {
                                report_error(p.err, kErrWaitTimeout, kWhereAttend, static_cast<int>(c), iter);
                                *abort_flag = 1;
                            }
                            abort = true;
                            break;
                        }
                        ++iter;
                    }
                }
            }
            gp = rs + j1;
        }
        if (abort && lane == 0) *abort_flag = 1;
        // Drain: every copy this warp issued has landed before the CTA can exit.
        if (lane == 0) {
            const int first = iter > NS ? iter - NS : 0;
            for (int it = first; it < iter; ++it) {
                if (!mbar_wait(&full[it % NS], static_cast<uint32_t>(it / NS) & 1u, kWaitLimitCycles)) {
                    report_error(p.err, kErrWaitTimeout, kWhereAttend, static_cast<int>(c), -it);
                    break;
                }
            }
        }
        return;
    }

    // ============ consumer warps: warps g and g + 8 <-> kv head g ============
    const int g = warp % kHkv;
    const int half = warp / kHkv;                   // alternate chunks: takes those with iter % 2 == half;
                                                    // token split: takes tokens [half * WT, half * WT + WT)
    const int qt = lane >> 3, j = lane & 7;
    const int k_idx = j >> KSHIFT;
    const int my_head = k_idx & 1;                   // which of the two q heads this lane's score is
    const int my_tok = qt * TPQ + (k_idx >> 1);      // token within the chunk
    float *my_p = pbuf + warp * (2 * CH);
    TOut *out = static_cast<TOut *>(p.out);

    if (p.early) pdl_wait();   // q and the merge scratch come from the preceding kernels
    int iter = 0;
    int nseg = 0;                                   // segments finished (both halves count alike)
    int r = r0;
    int64_t gp = pb;
    bool abort = false;
    while (gp < pe && !abort) {
        while (row_start[r + 1] <= gp) ++r;
        const int rs = row_start[r];
        const int re = row_start[r + 1];
        const int j0 = static_cast<int>(gp - rs);
        const int j1 = static_cast<int>((pe < re ? pe : re) - rs);
        const int len = p.lens[r];

        // q of heads 2g (a) and 2g+1 (b) for this lane's QK dims, pre-scaled.
        float qa[NC * E], qb[NC * E];
        {
            const float *qrow = p.q + static_cast<size_t>(r) * kQDim + (2 * g) * kHeadDim;
#pragma unroll
            for (int cc = 0; cc < NC; ++cc) {
#pragma unroll
                for (int e = 0; e < E; e += 4) {
                    const int d = (j + 8 * cc) * E + e;
                    const float4 a = *reinterpret_cast<const float4 *>(qrow + d);
                    const float4 b = *reinterpret_cast<const float4 *>(qrow + kHeadDim + d);
                    qa[cc * E + e + 0] = a.x * p.scale_log2; qa[cc * E + e + 1] = a.y * p.scale_log2;
                    qa[cc * E + e + 2] = a.z * p.scale_log2; qa[cc * E + e + 3] = a.w * p.scale_log2;
                    qb[cc * E + e + 0] = b.x * p.scale_log2; qb[cc * E + e + 1] = b.y * p.scale_log2;
                    qb[cc * E + e + 2] = b.z * p.scale_log2; qb[cc * E + e + 3] = b.w * p.scale_log2;
                }
            }
        }
        // e4m3 cache: q as f16 pairs for the mixed-precision dot (f16 x f16 -> f32).
        uint32_t qa2[kFp8 ? 8 : 1], qb2[kFp8 ? 8 : 1];
        if constexpr (kFp8) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                qa2[i] = pack_h2(qa[2 * i], qa[2 * i + 1]);
                qb2[i] = pack_h2(qb[2 * i], qb[2 * i + 1]);
            }
        }
        float m_run = -INFINITY, l_run = 0.0f;
        float oa[4] = {0.f, 0.f, 0.f, 0.f}, ob[4] = {0.f, 0.f, 0.f, 0.f};

        for (int jp = j0; jp < j1 && !abort; ++jp) {
#pragma unroll 1
            for (int cp = 0; cp < CPP; ++cp) {
                if (!kTSplit && iter % kHalves != half) {   // the partner warp takes this chunk
                    ++iter;
                    continue;
                }
                const int s = iter % NS;
                const uint32_t ph = static_cast<uint32_t>(iter / NS) & 1u;
                if (!stage_wait(&full[s], ph, abort_flag)) {
                    if (lane == 0) {
                        report_error(p.err, kErrWaitTimeout, kWhereAttend, static_cast<int>(c), iter);
                        *abort_flag = 1;
                    }
                    abort = true;
                    break;
                }
                const int wt0 = kTSplit ? half * WT : 0;    // first token of this warp's share
                const int tok0 = jp * kPageTokens + cp * CH + wt0;
                const int nvalid = len - tok0 < WT ? len - tok0 : WT;
                if (nvalid > 0) {
                    const TC *kst = stages + static_cast<size_t>(s) * (2 * HALF) + (g * CH + wt0) * kHeadDim;
                    const TC *vst = kst + HALF;
                    // 8-bit caches: the lane's token's K scale, and its V scale as a
                    // ratio to the largest V scale of the chunk's valid tokens (the
                    // ratio goes into p, the largest scale multiplies the chunk's sum).
                    float sk = 1.0f, sv = 1.0f, sv_ratio = 1.0f;
                    if constexpr (kFp8) {
                        const float *ss = sscale + s * kPageScales + g * kPageTokens;
                        sk = ss[my_tok];
                        const float sv_t = my_tok < nvalid ? ss[kHkv * kPageTokens + my_tok] : 0.0f;
                        sv = sv_t;
#pragma unroll
                        for (int o = 1; o < 32; o <<= 1) {
                            if (o != HB) sv = fmaxf(sv, __shfl_xor_sync(0xffffffffu, sv, o));
                        }
                        sv_ratio = sv > 0.0f ? __fdividef(sv_t, sv) : 0.0f;
                    }
                    // ---- QK ----
                    float part[NV];
#pragma unroll
                    for (int t = 0; t < TPQ; ++t) {
                        const TC *krow = kst + (qt * TPQ + t) * kHeadDim;
                        float acc_a = 0.f, acc_b = 0.f;
                        if constexpr (kFp8) {
                            // 16 e4m3 -> 8 f16x2 (exact), two mixed-precision FMAs per pair and head.
                            const uint4 w = *reinterpret_cast<const uint4 *>(krow + j * 16);
                            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                uint32_t x, y;
                                e4m3x4_to_h2x2(ws[k], x, y);
                                dot2_f16_f32(acc_a, qa2[2 * k], x);
                                dot2_f16_f32(acc_a, qa2[2 * k + 1], y);
                                dot2_f16_f32(acc_b, qb2[2 * k], x);
                                dot2_f16_f32(acc_b, qb2[2 * k + 1], y);
                            }
                        } else {
#pragma unroll
                            for (int cc = 0; cc < NC; ++cc) {
                                float kv[E];
                                Chunk16<TC>::load(krow + (j + 8 * cc) * E, kv);
#pragma unroll
                                for (int e = 0; e < E; ++e) {
                                    acc_a = fmaf(qa[cc * E + e], kv[e], acc_a);
                                    acc_b = fmaf(qb[cc * E + e], kv[e], acc_b);
                                }
                            }
                        }
                        part[2 * t + 0] = acc_a;
                        part[2 * t + 1] = acc_b;
                    }
                    reduce_scatter8<NV>(part, j);
                    float sc = part[0] * sk;
                    if (my_tok >= nvalid) sc = -INFINITY;
                    // ---- online softmax (per head, over the lanes of that head) ----
                    float mx = sc;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        if (o != HB) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    }
                    const float m_new = fmaxf(m_run, mx);
                    const float pv = exp2f(sc - m_new);
                    const float alpha = exp2f(m_run - m_new);
                    float ps = pv;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        if (o != HB && !(KSHIFT == 1 && o == 1)) ps += __shfl_xor_sync(0xffffffffu, ps, o);
                    }
                    l_run = l_run * alpha + ps;
                    m_run = m_new;
                    if constexpr (kFp8) {
                        reinterpret_cast<__half *>(my_p)[my_head * CH + my_tok] = __float2half_rn(pv * sv_ratio);
                    } else {
                        my_p[my_head * CH + my_tok] = pv;
                    }
                    const float al_a = __shfl_sync(0xffffffffu, alpha, 0);
                    const float al_b = __shfl_sync(0xffffffffu, alpha, HB);
                    __syncwarp();
                    // ---- PV ----
                    if constexpr (kFp8) {
                        // p (f16) x V (e4m3 or int8 -> f16x2, exact) accumulated in f32
                        // for this chunk (= one page), then scaled by the page's V scale once.
                        float xa[4] = {0.f, 0.f, 0.f, 0.f}, xb[4] = {0.f, 0.f, 0.f, 0.f};
                        const uint16_t *phalf = reinterpret_cast<const uint16_t *>(my_p);
                        // One token of V for this lane's 4 dims, both heads.
                        auto pv_token = [&](int t, uint32_t wa, uint32_t wb, int hsel) {
                            const uint32_t w = *reinterpret_cast<const uint32_t *>(vst + t * kHeadDim + 4 * lane);
                            uint32_t x, y;
                            if constexpr (kVI8) u8x4_to_h2x2(w, x, y);
                            else e4m3x4_to_h2x2(w, x, y);
                            if (hsel) {
                                axpy2_f16_f32<1>(xa[0], xa[1], x, wa); axpy2_f16_f32<1>(xa[2], xa[3], y, wa);
                                axpy2_f16_f32<1>(xb[0], xb[1], x, wb); axpy2_f16_f32<1>(xb[2], xb[3], y, wb);
                            } else {
                                axpy2_f16_f32<0>(xa[0], xa[1], x, wa); axpy2_f16_f32<0>(xa[2], xa[3], y, wa);
                                axpy2_f16_f32<0>(xb[0], xb[1], x, wb); axpy2_f16_f32<0>(xb[2], xb[3], y, wb);
                            }
                        };
                        if (nvalid == WT) {     // full page: no per-token guard
#pragma unroll
                            for (int t4 = 0; t4 < WT; t4 += 4) {
                                const uint2 pa = *reinterpret_cast<const uint2 *>(phalf + t4);
                                const uint2 pb = *reinterpret_cast<const uint2 *>(phalf + CH + t4);
                                pv_token(t4 + 0, pa.x, pb.x, 0);
                                pv_token(t4 + 1, pa.x, pb.x, 1);
                                pv_token(t4 + 2, pa.y, pb.y, 0);
                                pv_token(t4 + 3, pa.y, pb.y, 1);
                            }
                        } else {
#pragma unroll
                            for (int t4 = 0; t4 < WT; t4 += 4) {
                                const uint2 pa = *reinterpret_cast<const uint2 *>(phalf + t4);
                                const uint2 pb = *reinterpret_cast<const uint2 *>(phalf + CH + t4);
                                if (t4 + 0 < nvalid) pv_token(t4 + 0, pa.x, pb.x, 0);
                                if (t4 + 1 < nvalid) pv_token(t4 + 1, pa.x, pb.x, 1);
                                if (t4 + 2 < nvalid) pv_token(t4 + 2, pa.y, pb.y, 0);
                                if (t4 + 3 < nvalid) pv_token(t4 + 3, pa.y, pb.y, 1);
                            }
                        }
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            oa[e] = fmaf(sv, xa[e], oa[e] * al_a);
                            ob[e] = fmaf(sv, xb[e], ob[e] * al_b);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            oa[e] *= al_a;
                            ob[e] *= al_b;
                        }
#pragma unroll
                        for (int t4 = 0; t4 < WT; t4 += 4) {
                            const float4 pa4 = *reinterpret_cast<const float4 *>(my_p + t4);
                            const float4 pb4 = *reinterpret_cast<const float4 *>(my_p + CH + t4);
                            const float pa[4] = {pa4.x, pa4.y, pa4.z, pa4.w};
                            const float pbv[4] = {pb4.x, pb4.y, pb4.z, pb4.w};
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const int t = t4 + u;
                                if (t < nvalid) {
                                    const float4 v = load4<TC>(vst + t * kHeadDim + 4 * lane);
                                    oa[0] = fmaf(pa[u], v.x, oa[0]); oa[1] = fmaf(pa[u], v.y, oa[1]);
                                    oa[2] = fmaf(pa[u], v.z, oa[2]); oa[3] = fmaf(pa[u], v.w, oa[3]);
                                    ob[0] = fmaf(pbv[u], v.x, ob[0]); ob[1] = fmaf(pbv[u], v.y, ob[1]);
                                    ob[2] = fmaf(pbv[u], v.z, ob[2]); ob[3] = fmaf(pbv[u], v.w, ob[3]);
                                }
                            }
                        }
                    }
                    __syncwarp();
                }
                if (lane == 0) mbar_arrive(&empty[s]);
                ++iter;
            }
        }
        if (abort) break;

        // ---- segment end ----
        float m_a = __shfl_sync(0xffffffffu, m_run, 0), m_b = __shfl_sync(0xffffffffu, m_run, HB);
        float l_a = __shfl_sync(0xffffffffu, l_run, 0), l_b = __shfl_sync(0xffffffffu, l_run, HB);
        if constexpr (kHalves > 1) {
            float *xol = xo + (g * 32 + lane) * 8;
            if (half == 1) {
                // Hand (m, l, O) to warp g once it has merged the previous segment.
                if (!flag_wait(&xack[g], nseg, abort_flag)) {
                    if (lane == 0) {
                        report_error(p.err, kErrWaitTimeout, kWhereAttend, static_cast<int>(c), -1000 - nseg);
                        *abort_flag = 1;
                    }
                    break;
                }
                *reinterpret_cast<float4 *>(xol) = make_float4(oa[0], oa[1], oa[2], oa[3]);
                *reinterpret_cast<float4 *>(xol + 4) = make_float4(ob[0], ob[1], ob[2], ob[3]);
                if (lane == 0) {
                    xml[g * 4 + 0] = m_a; xml[g * 4 + 1] = l_a; xml[g * 4 + 2] = m_b; xml[g * 4 + 3] = l_b;
                }
                __threadfence_block();
                __syncwarp();
                if (lane == 0) xseq[g] = nseg + 1;
                ++nseg;
                gp = rs + j1;
                continue;
            }
            if (!flag_wait(&xseq[g], nseg + 1, abort_flag)) {
                if (lane == 0) {
                    report_error(p.err, kErrWaitTimeout, kWhereAttend, static_cast<int>(c), -2000 - nseg);
                    *abort_flag = 1;
                }
                break;
            }
            __threadfence_block();
            const float4 xa = *reinterpret_cast<const float4 *>(xol);
            const float4 xb = *reinterpret_cast<const float4 *>(xol + 4);
            const float m1a = xml[g * 4 + 0], l1a = xml[g * 4 + 1], m1b = xml[g * 4 + 2], l1b = xml[g * 4 + 3];
            __syncwarp();
            if (lane == 0) xack[g] = nseg + 1;
            const float Ma = fmaxf(m_a, m1a), Mb = fmaxf(m_b, m1b);
            // A half that took no chunk of this segment has m = -inf: its weight is 0.
            const float s0a = m_a == -INFINITY ? 0.f : exp2f(m_a - Ma), s1a = m1a == -INFINITY ? 0.f : exp2f(m1a - Ma);
            const float s0b = m_b == -INFINITY ? 0.f : exp2f(m_b - Mb), s1b = m1b == -INFINITY ? 0.f : exp2f(m1b - Mb);
            oa[0] = oa[0] * s0a + xa.x * s1a; oa[1] = oa[1] * s0a + xa.y * s1a;
            oa[2] = oa[2] * s0a + xa.z * s1a; oa[3] = oa[3] * s0a + xa.w * s1a;
            ob[0] = ob[0] * s0b + xb.x * s1b; ob[1] = ob[1] * s0b + xb.y * s1b;
            ob[2] = ob[2] * s0b + xb.z * s1b; ob[3] = ob[3] * s0b + xb.w * s1b;
            l_a = l_a * s0a + l1a * s1a;
            l_b = l_b * s0b + l1b * s1b;
            m_a = Ma;
            m_b = Mb;
        }
        ++nseg;
        const int64_t c0 = cta_of_page(rs, T, G);
        const int64_t c1 = cta_of_page(re - 1, T, G);
        TOut *orow = out + static_cast<size_t>(r) * kQDim + (2 * g) * kHeadDim + 4 * lane;
        if (c0 == c1) {
            const float ia = 1.0f / l_a, ib = 1.0f / l_b;
            store4<TOut>(orow, make_float4(oa[0] * ia, oa[1] * ia, oa[2] * ia, oa[3] * ia));
            store4<TOut>(orow + kHeadDim, make_float4(ob[0] * ib, ob[1] * ib, ob[2] * ib, ob[3] * ib));
        } else {
            const size_t slot_idx = static_cast<size_t>(r) + static_cast<size_t>(c);
            float *po = p.part_o + (slot_idx * kHq + 2 * g) * kHeadDim + 4 * lane;
            *reinterpret_cast<float4 *>(po) = make_float4(oa[0], oa[1], oa[2], oa[3]);
            *reinterpret_cast<float4 *>(po + kHeadDim) = make_float4(ob[0], ob[1], ob[2], ob[3]);
            if (lane == 0) {
                float *pml = p.part_ml + (slot_idx * kHq + 2 * g) * 2;
                pml[0] = m_a; pml[1] = l_a; pml[2] = m_b; pml[3] = l_b;
            }
            __threadfence();
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                const int old = atomicAdd(&p.counters[r * kHkv + g], 1);
                last = (old == static_cast<int>(c1 - c0));
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
                float M_a = -INFINITY, M_b = -INFINITY;
                for (int64_t cc = c0; cc <= c1; ++cc) {
                    const float *pml = p.part_ml + ((static_cast<size_t>(r) + cc) * kHq + 2 * g) * 2;
                    M_a = fmaxf(M_a, __ldcg(pml + 0));
                    M_b = fmaxf(M_b, __ldcg(pml + 2));
                }
                float4 A = make_float4(0.f, 0.f, 0.f, 0.f), B = A;
                float La = 0.f, Lb = 0.f;
                for (int64_t cc = c0; cc <= c1; ++cc) {
                    const size_t si = static_cast<size_t>(r) + static_cast<size_t>(cc);
                    const float *pml = p.part_ml + (si * kHq + 2 * g) * 2;
                    const float wa = exp2f(__ldcg(pml + 0) - M_a), wb = exp2f(__ldcg(pml + 2) - M_b);
                    La += wa * __ldcg(pml + 1);
                    Lb += wb * __ldcg(pml + 3);
                    const float *pp = p.part_o + (si * kHq + 2 * g) * kHeadDim + 4 * lane;
                    const float4 x = __ldcg(reinterpret_cast<const float4 *>(pp));
                    const float4 y = __ldcg(reinterpret_cast<const float4 *>(pp + kHeadDim));
                    A.x += wa * x.x; A.y += wa * x.y; A.z += wa * x.z; A.w += wa * x.w;
                    B.x += wb * y.x; B.y += wb * y.y; B.z += wb * y.z; B.w += wb * y.w;
                }
                const float ia = 1.0f / La, ib = 1.0f / Lb;
                store4<TOut>(orow, make_float4(A.x * ia, A.y * ia, A.z * ia, A.w * ia));
                store4<TOut>(orow + kHeadDim, make_float4(B.x * ib, B.y * ib, B.z * ib, B.w * ib));
                if (lane == 0) p.counters[r * kHkv + g] = 0;
            }
        }
        gp = rs + j1;
    }
}

template <typename TC, typename TOut, bool kVI8 = false> cudaError_t prepare_t() {
    return cudaFuncSetAttribute(decode_attn_kernel<TC, TOut, kVI8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem_bytes<TC>()));
}

template <typename TC, typename TOut, bool kVI8 = false>
cudaError_t launch_t(const AttendParams &p, int grid, cudaStream_t st) {
    return launch_pdl(decode_attn_kernel<TC, TOut, kVI8>, dim3(grid), dim3(threads<TC>()), smem_bytes<TC>(), st, p);
}

}  // namespace

// Opt the kernels into > 48 KB of dynamic shared memory on the current device.
cudaError_t prepare_decode_attn() {
    cudaError_t e;
    if ((e = prepare_t<float, float>()) != cudaSuccess) return e;
    if ((e = prepare_t<float, __nv_bfloat16>()) != cudaSuccess) return e;
    if ((e = prepare_t<__nv_bfloat16, float>()) != cudaSuccess) return e;
    if ((e = prepare_t<__nv_bfloat16, __nv_bfloat16>()) != cudaSuccess) return e;
    if ((e = prepare_t<uint8_t, float>()) != cudaSuccess) return e;
    if ((e = prepare_t<uint8_t, __nv_bfloat16>()) != cudaSuccess) return e;
    if ((e = prepare_t<uint8_t, float, true>()) != cudaSuccess) return e;
    return prepare_t<uint8_t, __nv_bfloat16, true>();
}

size_t attn_smem_bytes(int kv_dtype) {
    switch (kv_dtype) {
        case kKvF32: return smem_bytes<float>();
        case kKvBF16: return smem_bytes<__nv_bfloat16>();
        case kKvFP8:
        case kKvE4I8: return smem_bytes<uint8_t>();
        default: return 0;
    }
}

cudaError_t launch_decode_attn(const AttendParams &p, int kv_dtype, bool out_bf16, int grid, cudaStream_t st) {
    if (p.n <= 0) return cudaSuccess;
    if (p.n > kAttnMaxRows) return cudaErrorInvalidValue;
    switch (kv_dtype) {
        case kKvF32: return out_bf16 ? launch_t<float, __nv_bfloat16>(p, grid, st) : launch_t<float, float>(p, grid, st);
        case kKvBF16:
            return out_bf16 ? launch_t<__nv_bfloat16, __nv_bfloat16>(p, grid, st) : launch_t<__nv_bfloat16, float>(p, grid, st);
        case kKvFP8: return out_bf16 ? launch_t<uint8_t, __nv_bfloat16>(p, grid, st) : launch_t<uint8_t, float>(p, grid, st);
        case kKvE4I8:
            return out_bf16 ? launch_t<uint8_t, __nv_bfloat16, true>(p, grid, st) : launch_t<uint8_t, float, true>(p, grid, st);
        default: return cudaErrorInvalidValue;
    }
}

namespace {

// Read probe: the ceiling of K2's page stream.  The same persistent grid and
// page split as K2 (CTA c of G takes pages [c n / G, (c + 1) n / G) of the
// list, which holds the rows' pages end to end in K2's order), each page's
// K and V block (page_bytes <= 64 KB, contiguous) brought into a 3-stage
// shared-memory ring by one cp.async.bulk copy from this GPU's own memory
// with the L2 evict-first hint, no multicast.  The consumer warp only waits
// for each stage to land and hands it back; nothing is computed.  Every wait
// is bounded, and the producer drains its copies before the CTA exits.
constexpr int kProbeStages = 3;
__global__ void __launch_bounds__(64, 1) page_read_probe_kernel(const uint8_t *pool, uint32_t page_bytes,
                                                                const int *pages, int n, int n_pool_pages,
                                                                DevError *err) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + static_cast<size_t>(kProbeStages) * page_bytes);
    uint64_t *empty = full + kProbeStages;
    __shared__ int never;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        never = 0;
        for (int s = 0; s < kProbeStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (lane != 0) return;
    const int64_t G = gridDim.x, c = blockIdx.x;
    const int p0 = static_cast<int>(c * n / G), p1 = static_cast<int>((c + 1) * n / G);
    if (warp == 0) {
        const uint64_t pol = l2_evict_first_policy();
        int iter = 0;
        for (int i = p0; i < p1; ++i, ++iter) {
            const int s = iter % kProbeStages;
            const uint32_t ph = static_cast<uint32_t>(iter / kProbeStages) & 1u;
            const int page = pages[i];
            if (page < 0 || page >= n_pool_pages) {
                report_error(err, kErrPageIndex, kWhereProbe, i, page);
                break;
            }
            if (!stage_wait(&empty[s], ph ^ 1u, &never)) {
                report_error(err, kErrWaitTimeout, kWhereProbe, static_cast<int>(c), iter);
                break;
            }
            mbar_arrive_expect_tx(&full[s], page_bytes);
            bulk_g2s(smem + static_cast<size_t>(s) * page_bytes, pool + static_cast<size_t>(page) * page_bytes,
                     page_bytes, &full[s], pol);
        }
        // Drain: every copy issued has landed before the CTA can exit.
        for (int it = iter > kProbeStages ? iter - kProbeStages : 0; it < iter; ++it) {
            if (!mbar_wait(&full[it % kProbeStages], static_cast<uint32_t>(it / kProbeStages) & 1u, kWaitLimitCycles)) {
                report_error(err, kErrWaitTimeout, kWhereProbe, static_cast<int>(c), -it);
                break;
            }
        }
    } else {
        for (int i = p0, iter = 0; i < p1; ++i, ++iter) {
            const int s = iter % kProbeStages;
            if (!stage_wait(&full[s], static_cast<uint32_t>(iter / kProbeStages) & 1u, &never)) {
                report_error(err, kErrWaitTimeout, kWhereProbe, static_cast<int>(c), iter);
                break;
            }
            mbar_arrive(&empty[s]);
        }
    }
}

}  // namespace

size_t page_read_probe_smem(uint32_t page_bytes) {
    return static_cast<size_t>(kProbeStages) * page_bytes + 2 * kProbeStages * sizeof(uint64_t);
}

cudaError_t launch_page_read_probe(const void *pool_layer, uint32_t page_bytes, const int *pages, int n,
                                   int n_pool_pages, int grid, DevError *err, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (page_bytes == 0 || page_bytes > 65536u || page_bytes % 16 != 0) return cudaErrorInvalidValue;
    const size_t smem = page_read_probe_smem(page_bytes);
    cudaError_t e = cudaFuncSetAttribute(page_read_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    page_read_probe_kernel<<<grid, 64, smem, st>>>(static_cast<const uint8_t *>(pool_layer), page_bytes, pages, n,
                                                    n_pool_pages, err);
    return cudaGetLastError();
}

cudaError_t launch_wait_probe(DevError *err, long long limit_cycles, cudaStream_t st) {
    wait_probe_kernel<<<1, 64, 0, st>>>(err, limit_cycles);
    return cudaGetLastError();
}

}  // namespace qkv

// ---------------------------------------------------------------------------
// Allocation-free variant of K2 for callers that may not allocate device
// memory themselves: code embedded in a host framework that owns every device
// buffer through its own allocator and memory plan (a GGML backend scheduler
// with pre-sized buffers, an inference server that budgets HBM up front), where
// a cudaMalloc/cudaFree behind the framework's back breaks its accounting or
// is simply not permitted.  Such a caller passes its own KV pool, page table,
// queries and output; the kernel's scratch (split-row partials, per-row merge
// counters, the device error word) comes from the file-scope array below,
// which every GPU that loads this library holds until the process exits.
// ---------------------------------------------------------------------------
namespace qkv {
namespace {

constexpr int kNoAllocMaxRows = 256;   // rows per call
constexpr int kNoAllocMaxGrid = 160;   // CTAs per call (B200 has 148 SMs)
constexpr size_t kNoAllocSlots = static_cast<size_t>(kNoAllocMaxRows + kNoAllocMaxGrid);
constexpr size_t kNoAllocOBytes = kNoAllocSlots * kHq * kHeadDim * sizeof(float);   // 3.4 MB
constexpr size_t kNoAllocMLBytes = kNoAllocSlots * kHq * 2 * sizeof(float);
constexpr size_t kNoAllocCntBytes = static_cast<size_t>(kNoAllocMaxRows) * kHkv * sizeof(int);
constexpr size_t kNoAllocBytes = kNoAllocOBytes + kNoAllocMLBytes + kNoAllocCntBytes + 256;

// Host code must not use this name as an address: on the host it is only a
// stand-in for the symbol.  The device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
uint8_t *g_noalloc_addr[kMaxDevices] = {};
int g_noalloc_sms[kMaxDevices] = {};

void noalloc_err(char *err, size_t len, const char *msg) {
    if (err && len > 0) {
        std::strncpy(err, msg, len - 1);
        err[len - 1] = '\0';
    }
}

// Once per device, with that device current: resolve the scratch array's
// device address, opt the kernels into their shared-memory size, read the SM
// count and clear the array.
int noalloc_setup(int dev, char *err, size_t err_len) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_addr[dev]) return QKV_OK;
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr) {
        noalloc_err(err, err_len, "cudaGetSymbolAddress(g_noalloc_scratch) failed");
        return QKV_ERR_CUDA;
    }
    int sms = 0;
    if ((e = prepare_decode_attn()) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaMemset(ptr, 0, kNoAllocBytes)) != cudaSuccess || (e = cudaDeviceSynchronize()) != cudaSuccess) {
        noalloc_err(err, err_len, cudaGetErrorString(e));
        return QKV_ERR_CUDA;
    }
    g_noalloc_sms[dev] = sms;
    g_noalloc_addr[dev] = static_cast<uint8_t *>(ptr);
    return QKV_OK;
}

}  // namespace
}  // namespace qkv

extern "C" int qkv_kv_attend_noalloc(const void *pool_layer, int32_t kv_dtype, const float *scales_layer,
                                     const int32_t *page_table, int32_t maxp, int32_t max_streams, int32_t n_pages,
                                     int32_t n, const int32_t *slots_dev, const int32_t *lens_dev, const float *q_dev,
                                     float *out_dev, void *stream, char *err, size_t err_len) {
    using namespace qkv;
    if (n < 0 || !pool_layer || !page_table || maxp <= 0 || max_streams <= 0 || n_pages <= 0 ||
        (n > 0 && (!slots_dev || !lens_dev || !q_dev || !out_dev)) || kv_dtype < kKvF32 || kv_dtype > kKvE4I8 ||
        (kv_is_8bit(kv_dtype) && !scales_layer)) {
        noalloc_err(err, err_len, "kv_attend_noalloc: bad argument");
        return QKV_ERR_INVALID_ARG;
    }
    if (n > kNoAllocMaxRows) {
        noalloc_err(err, err_len, "kv_attend_noalloc: more than 256 rows in one call (the fixed scratch limit)");
        return QKV_ERR_CAPACITY;
    }
    if (n == 0) return QKV_OK;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        noalloc_err(err, err_len, "kv_attend_noalloc: no current CUDA device");
        return QKV_ERR_NO_DEVICE;
    }
    int rc = noalloc_setup(dev, err, err_len);
    if (rc != QKV_OK) return rc;
    uint8_t *base = g_noalloc_addr[dev];
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    AttendParams p{};
    p.n = n;
    p.slots = slots_dev;
    p.lens = lens_dev;
    p.q = q_dev;
    p.out = out_dev;
    p.pool = pool_layer;
    p.scales = scales_layer;
    p.page_table = page_table;
    p.maxp = maxp;
    p.max_streams = max_streams;
    p.n_pages = n_pages;
    p.part_o = reinterpret_cast<float *>(base);
    p.part_ml = reinterpret_cast<float *>(base + kNoAllocOBytes);
    p.counters = reinterpret_cast<int *>(base + kNoAllocOBytes + kNoAllocMLBytes);
    p.err = reinterpret_cast<DevError *>(base + kNoAllocOBytes + kNoAllocMLBytes + kNoAllocCntBytes);
    p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(kHeadDim)));
    // The merge counters must start at zero (a call that stopped early, when a
    // bounded wait ran out, could have left some set), and the error word
    // directly after them is cleared too, so no earlier call's error stays
    // latched in the shared array.  This entry never reads the word back: a
    // read would need a synchronisation the caller has not asked for.
    cudaError_t e = cudaMemsetAsync(p.counters, 0, kNoAllocCntBytes + sizeof(DevError), st);
    const int grid = g_noalloc_sms[dev] < kNoAllocMaxGrid ? g_noalloc_sms[dev] : kNoAllocMaxGrid;
    if (e == cudaSuccess) e = launch_decode_attn(p, kv_dtype, false, grid, st);
    if (e != cudaSuccess) {
        noalloc_err(err, err_len, cudaGetErrorString(e));
        return QKV_ERR_CUDA;
    }
    return QKV_OK;
}
