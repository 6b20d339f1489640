// K3: causal prefill attention on the tensor cores (tcgen05 + TMEM) over the
// paged cache, bf16 or e4m3.  Replaces the prompt half of
// text-decoder.cpp:322-334 (QK^T, diag mask, softmax, PV over the whole
// prompt) for the paged cache that K1 has just filled (and the scalar twin
// :739-791).
//
// One CTA per work item = (64 consecutive queries of one stream, kv head g).
// GQA: the two q heads of kv head g share the item, so the MMA's M = 128 rows
// are [64 queries of head 2g | 64 queries of head 2g+1] and every K/V tile is
// fetched once for both.  Keys come in tiles of 128 (8 pages).
//
// Operand staging: a warpgroup of 128 loader threads reads each tile's key rows
// straight from their pages with coalesced 16-byte loads (16 lanes per bf16
// row, 8 per e4m3 row) and writes them into the canonical 128-byte-swizzled
// UMMA layout — K as the K-major B operand of
// S = Q K^T, V as the MN-major B operand of O += P V.  (A page contributes
// 16 scattered rows per head; one TMA copy per page and column block would be
// bounded by the rate at which a thread can issue copies.)  For the e4m3 cache
// the loader dequantises on the way (e4m3 -> f16 exactly, times the page's
// per-(kv, head) scale in f16), and Q, P are f16 too; for bf16 everything is
// bf16.  K and V tiles are double-buffered, S is double-buffered in TMEM.
//
// One pass over the key tiles with an online softmax: the issuer puts S of
// tile t + 1 ahead of P V of tile t (across items too: the next item's first S
// goes ahead of this item's last P V), so the softmax of a tile overlaps the
// MMAs around it.  P is written unnormalised against a per-row reference max;
// the reference moves (and O, l are rescaled in place in TMEM) only when a
// tile's max exceeds it by more than 2^8, so P stays within [0, 256] and most
// tiles need no correction; O is divided by the row sum in the epilogue.
//
// Roles: warps 0..3 loaders, warps 4..11 softmax/epilogue in two warpgroups
// that split each row's key columns (thread = TMEM lane = one query row; lane
// quadrant = warp % 4), warp 12 TMEM allocator + MMA issuer (one thread).
// All waits bounded.
#include "kernels.h"

namespace qkv {

namespace {

constexpr int kQPerItem = 64;
constexpr int kKeyTile = 128;
constexpr uint32_t kBlkBytes = 128 * 128;                 // [128 rows][64 x 16-bit], 16 KB
constexpr uint32_t kTileBytes = 2 * kBlkBytes;            // two 64-column blocks, 32 KB
constexpr int kSoftmaxWarp0 = 4;                          // warps 4..11: two softmax warpgroups
constexpr int kMmaWarp = 12;
constexpr int kThreads = 13 * 32;
// Shared memory from a 1024-byte boundary: Q[2], K[2], V[2], P tiles, then the
// row hand-over ring [2 slots][2 halves][128 rows] of floats, the barriers,
// the TMEM address and the abort flag.
constexpr size_t kTiles = 7;
constexpr size_t kXBytes = 2 * 2 * 128 * sizeof(float);
constexpr size_t kTailBytes = kXBytes + 256;
constexpr size_t kSmemNeed = kTiles * static_cast<size_t>(kTileBytes) + kTailBytes;
constexpr float kRescaleLog2 = 8.0f;                       // P <= 2^8 between reference moves
constexpr uint32_t kTmemCols = 512;                       // S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512)
constexpr uint32_t kTmemO = 256;

struct K3Params {
    const int4 *items;      // (row0, nq, g, 0)
    const int *slots;
    const int *positions;
    const uint16_t *q16;    // [rows][2048] post-RoPE q x scale_log2, bf16 (f16 for e4m3)
    void *out;              // [rows][2048]
    int out_bf16;
    const void *pool;
    const float *scales;    // 8-bit caches: [pages][2][8][16]
    const int *page_table;
    int maxp;
    int max_streams;
    int n_pages;
    DevError *err;
    int v_int8;             // 8-bit cache: V tiles are int8 (excess-128 bytes), not e4m3
};

// Swizzled (128 B) operand descriptors, sm_100 version bit set.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t addr) {
    return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | ((1024ull >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// MN-major tile: 64-element MN blocks kBlkBytes apart (LBO), 8-row K groups 1024 B apart (SBO).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t addr) {
    return ((addr >> 4) & 0x3FFFull) | (static_cast<uint64_t>(kBlkBytes >> 4) << 16) | ((1024ull >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}

// Instruction descriptors: f32 accumulate, A and B both bf16 (bits 7, 10) or
// both f16, M = 128, N = 128; PV takes B (V) MN-major (bit 16).
template <bool F16> constexpr uint32_t idesc_s() {
    return (1u << 4) | (F16 ? 0u : ((1u << 7) | (1u << 10))) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
}
template <bool F16> constexpr uint32_t idesc_pv() { return idesc_s<F16>() | (1u << 16); }

__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, int acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive TMEM columns of this thread's lane; the values are usable
// after tmem_wait_ld().
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
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

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    tmem_ld32_issue(taddr, r);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive TMEM columns of this thread's lane; ordered by tmem_wait_st().
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2^x by the SFU's approximate instruction (PTX ex2.approx.ftz.f32): denormal
// results flush to zero, 2^-inf = 0.  P is rounded to 16 bits right after, so
// neither the approximation nor the flush is visible in it.
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Byte offset of 16-byte chunk c (0..7) of row r inside a 128B-swizzled block.
__device__ __forceinline__ uint32_t swz(int r, int c) {
    return static_cast<uint32_t>(r) * 128u + (static_cast<uint32_t>(c ^ (r & 7)) << 4);
}

template <bool F16> __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if constexpr (F16) return pack_h2(lo, hi);
    else return pack_bf16x2(lo, hi);
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t s2) {
    __half2 x, y;
    memcpy(&x, &a, 4);
    memcpy(&y, &s2, 4);
    const __half2 z = __hmul2(x, y);
    uint32_t r;
    memcpy(&r, &z, 4);
    return r;
}

// 16-byte asynchronous global -> shared copy (L2 only); src_bytes 0 writes zeros.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
// Arrive on `bar` once every cp.async this thread issued so far has landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Page ids of key tile kt's 8 pages (clamped past the stream's last page).
__device__ __forceinline__ void tile_pages(const int *pt, int key_pages, int kt, int (&pg)[8]) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int pi = kt * 8 + k;
        pg[k] = __ldg(pt + (pi < key_pages ? pi : 0));
    }
}

// bf16 tile by cp.async, straight into the swizzled layout: thread t copies
// 16-byte chunk t % 16 of rows t / 16 + 8m (row r0 + 8m lies in page m / 2);
// dead keys are zero-filled by the copy itself.
__device__ __forceinline__ bool copy_tile_async(const K3Params &p, uint8_t *tile, const int (&pg)[8], int kv_len, int kt,
                                                int kv, int g, int t) {
    const int c = t & 15, r0 = t >> 4;
    bool ok = true;
#pragma unroll
    for (int m = 0; m < 16; ++m) {
        const int r = r0 + 8 * m;
        const int key = kt * kKeyTile + r;
        const bool live = key < kv_len;
        const int page = pg[m >> 1];
        const bool valid = page >= 0 && page < p.n_pages;
        if (live && !valid) ok = false;
        const size_t row = ((static_cast<size_t>(valid ? page : 0) * 2 + kv) * kHkv + g) * kPageTokens + key % kPageTokens;
        const uint8_t *src = static_cast<const uint8_t *>(p.pool) + row * kHeadDim * 2 + c * 16;
        cp_async16(tile + (c >> 3) * kBlkBytes + swz(r, c & 7), src, (live && valid) ? 16u : 0u);
    }
    return ok;
}

// Tile loading, coalesced: the 128 loader threads cover a tile's 128 key rows
// chunk-wise — for bf16, thread t reads 16-byte chunk t % 16 of rows
// t / 16 + 8m (m = 0..15), so 16 lanes read one 256-byte row; for e4m3, chunk
// t % 8 of rows t / 8 + 16m (m = 0..7), 8 lanes per 128-byte row.  Keys past
// the stream's length are not read and store as zeros.
template <typename TC> struct TileRegs {
    static constexpr int kChunks = sizeof(TC) == 2 ? 16 : 8;   // per row
    static constexpr int kRows = 128 * kChunks / 128;          // rows per thread: 16 (bf16) or 8 (e4m3)
    static constexpr int kStride = 128 / kRows;                // row step between a thread's rows
    uint4 w[kRows];
    uint32_t live;                                             // bit m: row m of this thread is a live key
};

// e4m3 tile into registers: thread t reads 16-byte chunk t % 8 of rows
// t / 8 + 16m (row r0 + 16m lies in page m).
template <typename TC>
__device__ __forceinline__ bool fetch_tile(const K3Params &p, TileRegs<TC> &tr, const int (&pg)[8], int kv_len, int kt,
                                           int kv, int g, int t) {
    static_assert(sizeof(TC) == 1, "register path is the e4m3 cache's");
    using TR = TileRegs<TC>;
    const int c = t % TR::kChunks, r0 = t / TR::kChunks;
    bool ok = true;
    tr.live = 0;
#pragma unroll
    for (int m = 0; m < TR::kRows; ++m) {
        const int key = kt * kKeyTile + r0 + TR::kStride * m;
        const bool live = key < kv_len;
        const bool valid = pg[m] >= 0 && pg[m] < p.n_pages;
        if (live) tr.live |= 1u << m;
        if (live && !valid) ok = false;
        const int page = valid ? pg[m] : 0;
        const size_t row = ((static_cast<size_t>(page) * 2 + kv) * kHkv + g) * kPageTokens + key % kPageTokens;
        tr.w[m] = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(p.pool) + row * kHeadDim) + c);
    }
#pragma unroll
    for (int m = 0; m < TR::kRows; ++m) {
        if (!((tr.live >> m) & 1u)) tr.w[m] = make_uint4(0, 0, 0, 0);
    }
    return ok;
}

// Into a swizzled [2 blocks][128 rows][64] 16-bit tile (8-bit cache: e4m3,
// or int8 for V tiles of the e4m3-K / int8-V cache, dequantised exactly to
// f16, then times the page's (kv, g) scale in f16, read here so it does not
// occupy registers while the loader waits for the buffer).
template <typename TC>
__device__ __forceinline__ void store_tile(const K3Params &p, uint8_t *tile, const TileRegs<TC> &tr, const int (&pg)[8],
                                           int kv, int g, int t) {
    using TR = TileRegs<TC>;
    const int c = t % TR::kChunks, r0 = t / TR::kChunks;
#pragma unroll
    for (int m = 0; m < TR::kRows; ++m) {
        const int r = r0 + TR::kStride * m;
        if constexpr (sizeof(TC) == 2) {
            *reinterpret_cast<uint4 *>(tile + (c >> 3) * kBlkBytes + swz(r, c & 7)) = tr.w[m];
        } else {
            // 16 e4m3 = dims 16c .. 16c+15 -> f16 chunks 2c (dims 16c..+7) and 2c+1
            const bool valid = pg[m] >= 0 && pg[m] < p.n_pages;
            // the row's own (token, head) scale; row r of the tile is token r % 16 of its page
            const float sc = __ldg(p.scales + ((static_cast<size_t>(valid ? pg[m] : 0) * 2 + kv) * kHkv + g) * kPageTokens +
                                   (r & (kPageTokens - 1)));
            const uint32_t s2 = pack_h2(sc, sc);
            const uint32_t ws[4] = {tr.w[m].x, tr.w[m].y, tr.w[m].z, tr.w[m].w};
            const bool i8 = kv == 1 && p.v_int8;
            uint32_t h[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                uint32_t lo2, hi2;
                if (i8) u8x4_to_h2x2(ws[k], lo2, hi2);
                else e4m3x4_to_h2x2(ws[k], lo2, hi2);
                h[2 * k] = hmul2_bits(lo2, s2);
                h[2 * k + 1] = hmul2_bits(hi2, s2);
            }
            const int c0 = 2 * c, c1 = 2 * c + 1;
            *reinterpret_cast<uint4 *>(tile + (c0 >> 3) * kBlkBytes + swz(r, c0 & 7)) = make_uint4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<uint4 *>(tile + (c1 >> 3) * kBlkBytes + swz(r, c1 & 7)) = make_uint4(h[4], h[5], h[6], h[7]);
        }
    }
}

struct Bars {
    uint64_t q_full[2], q_empty[2], k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], s_free[2];
    uint64_t p_full, p_free, o_full[2], o_empty[2], x_ready[2], mma_done;
};
static_assert(sizeof(Bars) + 2 * sizeof(uint32_t) <= kTailBytes - kXBytes, "tail of the shared-memory layout");

// Bounded wait that also gives up as soon as another role set the abort flag.
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *failed) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*failed) return false;
        if (clock64() - t0 > kWaitLimitCycles) return false;
    }
    return true;
}

struct ItemInfo {
    int row0, nq, g, slot, pos0, kv_len, n_kt, key_pages;
    bool ok;
};

__device__ __forceinline__ ItemInfo item_info(const K3Params &p, int it) {
    const int4 v = p.items[it];
    ItemInfo f;
    f.row0 = v.x;
    f.nq = v.y;
    f.g = v.z;
    f.slot = p.slots[f.row0];
    f.pos0 = p.positions[f.row0];
    f.kv_len = f.pos0 + f.nq;
    f.n_kt = (f.kv_len + kKeyTile - 1) / kKeyTile;
    f.key_pages = (f.kv_len + kPageTokens - 1) / kPageTokens;
    f.ok = f.slot >= 0 && f.slot < p.max_streams && f.pos0 >= 0 && f.nq > 0 && f.nq <= kQPerItem &&
           f.key_pages <= p.maxp && f.g >= 0 && f.g < kHkv;
    return f;
}

// Persistent: CTA c takes items c, c + G, c + 2G, ... (the host puts the
// items of one (stream, kv head) pair back to back, longest first, so a pair's
// query blocks run together on neighbouring CTAs and share its K/V in L2).  Every barrier phase follows from per-role counters that
// run on across items: item j uses the Q tile and O buffer j & 1; key tile u
// (global count) uses K, V and S buffers u & 1 and the single P tile; the
// softmax threads' x-th row hand-over (each tile's max, each item's sum) uses
// ring slot x & 1.
// 13 warps: the SM's four sub-partitions hold up to 4 of them each, which caps
// a thread at 128 registers.
template <typename TC>
__global__ void __launch_bounds__(kThreads, 1) prefill_attn_tc_kernel(K3Params p, int n_items) {
    constexpr bool kF16 = sizeof(TC) == 1;   // e4m3 cache -> f16 operands
    extern __shared__ uint8_t smem_raw[];
    pdl_trigger();
    // The tiles need a 1024-byte boundary; the layout must fit the launch's allocation.
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint32_t dyn_bytes;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_bytes));
    if (static_cast<size_t>(smem - smem_raw) + kSmemNeed > dyn_bytes) {
        if (threadIdx.x == 0) report_error(p.err, kErrRowBounds, kWherePrefillAttn, -1, static_cast<int>(dyn_bytes));
        return;
    }
    uint8_t *const sQ0 = smem;                       // Q[b] = sQ0 + b * kTileBytes
    uint8_t *const sK0 = smem + 2 * kTileBytes;      // K[b]
    uint8_t *const sV0 = smem + 4 * kTileBytes;      // V[b]
    uint8_t *const sP = smem + 6 * kTileBytes;
    float *const xr = reinterpret_cast<float *>(smem + kTiles * kTileBytes);   // row hand-over [slot][half][row]
    Bars *bars = reinterpret_cast<Bars *>(smem + kTiles * kTileBytes + kXBytes);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 1);
    volatile int *failed = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->q_full[b], 128);
            mbar_init(&bars->q_empty[b], 1);
            mbar_init(&bars->k_full[b], 128);
            mbar_init(&bars->k_empty[b], 1);
            mbar_init(&bars->v_full[b], 128);
            mbar_init(&bars->v_empty[b], 1);
            mbar_init(&bars->s_full[b], 1);
            mbar_init(&bars->s_free[b], 256);
            mbar_init(&bars->o_full[b], 1);
            mbar_init(&bars->o_empty[b], 256);
            mbar_init(&bars->x_ready[b], 256);
        }
        mbar_init(&bars->p_full, 256);
        mbar_init(&bars->p_free, 1);
        mbar_init(&bars->mma_done, 1);
        *failed = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();   // items, q rows and the pages come from earlier kernels and copies

    if (warp < 4) {
        // ================= loaders: Q rows, then K/V tiles chunk-wise =================
        const int r = threadIdx.x;
        uint32_t ku = 0, j = 0;
        for (int it = blockIdx.x; it < n_items && !*failed; it += gridDim.x, ++j) {
            const ItemInfo f = item_info(p, it);
            if (!f.ok) {
                if (r == 0) report_error(p.err, kErrRowBounds, kWherePrefillAttn, f.row0, f.pos0);
                *failed = 1;
                break;
            }
            const int *pt = p.page_table + static_cast<size_t>(f.slot) * p.maxp;
            {
                // Q rows (head 2g + h, query i) -> tile row (h << 6) | i, swizzled K-major,
                // by cp.async like a key tile: thread t copies 16-byte chunk t % 16 of rows
                // t / 16 + 8m; rows past the item's queries are zero-filled.
                const uint32_t qb = j & 1;
                if (!wait_bar(&bars->q_empty[qb], ((j >> 1) & 1u) ^ 1u, failed)) {
                    if (!*failed) report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, f.row0, -(1 << 20));
                    *failed = 1;
                    break;
                }
                uint8_t *q_tile = sQ0 + qb * kTileBytes;
                const int c = r & 15;
#pragma unroll
                for (int m = 0; m < 16; ++m) {
                    const int row = (r >> 4) + 8 * m, h = row >> 6, i = row & 63;
                    const bool live = i < f.nq;
                    const uint16_t *src =
                        p.q16 + static_cast<size_t>(f.row0 + (live ? i : 0)) * kQDim + (2 * f.g + h) * kHeadDim + 8 * c;
                    cp_async16(q_tile + (c >> 3) * kBlkBytes + swz(row, c & 7), src, live ? 16u : 0u);
                }
                cp_async_arrive(&bars->q_full[qb]);
            }
            bool bad = false;
            int pg[8], pg_next[8];
            tile_pages(pt, f.key_pages, 0, pg);
            for (int kt = 0; kt < f.n_kt; ++kt) {
                const uint32_t kb = ku & 1, par = ((ku >> 1) & 1u) ^ 1u;
                // next tile's page ids in flight while this tile's copies are issued
                if (kt + 1 < f.n_kt) tile_pages(pt, f.key_pages, kt + 1, pg_next);
                if constexpr (sizeof(TC) == 2) {
                    // bf16: asynchronous copies; the loader runs ahead as far as the buffers allow.
                    if (!wait_bar(&bars->k_empty[kb], par, failed)) {
                        if (!*failed) report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, f.row0, kt);
                        *failed = 1;
                        bad = true;
                        break;
                    }
                    bool ok = copy_tile_async(p, sK0 + kb * kTileBytes, pg, f.kv_len, kt, 0, f.g, r);
                    cp_async_arrive(&bars->k_full[kb]);
                    if (!wait_bar(&bars->v_empty[kb], par, failed)) {
                        if (!*failed) report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, f.row0, -1 - kt);
                        *failed = 1;
                        bad = true;
                        break;
                    }
                    ok = copy_tile_async(p, sV0 + kb * kTileBytes, pg, f.kv_len, kt, 1, f.g, r) && ok;
                    cp_async_arrive(&bars->v_full[kb]);
                    ++ku;
                    if (!ok) {
                        report_error(p.err, kErrPageIndex, kWherePrefillAttn, f.row0, kt);
                        *failed = 1;
                        bad = true;
                        break;
                    }
                } else {
                    // e4m3: K and V loads in flight together, dequantised on the way in.
                    TileRegs<TC> kr, vr;
                    bool ok = fetch_tile<TC>(p, kr, pg, f.kv_len, kt, 0, f.g, r);
                    ok = fetch_tile<TC>(p, vr, pg, f.kv_len, kt, 1, f.g, r) && ok;
                    if (!ok) {
                        report_error(p.err, kErrPageIndex, kWherePrefillAttn, f.row0, kt);
                        *failed = 1;
                        bad = true;
                        break;
                    }
                    if (!wait_bar(&bars->k_empty[kb], par, failed)) {
                        if (!*failed) report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, f.row0, kt);
                        *failed = 1;
                        bad = true;
                        break;
                    }
                    store_tile<TC>(p, sK0 + kb * kTileBytes, kr, pg, 0, f.g, r);
                    fence_async_smem();
                    mbar_arrive(&bars->k_full[kb]);
                    if (!wait_bar(&bars->v_empty[kb], par, failed)) {
                        if (!*failed) report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, f.row0, -1 - kt);
                        *failed = 1;
                        bad = true;
                        break;
                    }
                    store_tile<TC>(p, sV0 + kb * kTileBytes, vr, pg, 1, f.g, r);
                    fence_async_smem();
                    mbar_arrive(&bars->v_full[kb]);
                    ++ku;
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) pg[k] = pg_next[k];
            }
            if (bad) break;
        }
        if constexpr (sizeof(TC) == 2) asm volatile("cp.async.wait_all;" ::: "memory");   // no copy outlives the CTA
    } else if (warp == kMmaWarp) {
        // ================= MMA issuer =================
        if (lane == 0) {
            bool ok = true, any = false;
            uint32_t ku = 0, j = 0;
            const uint32_t aP = smem_u32(sP);
            // P V of a tile is issued after S of the next tile in the CTA's stream,
            // the next item's first tile included, so S is ready when the softmax
            // threads come back from an item's epilogue.
            struct Pending {
                bool live;
                bool last;        // the item's last key tile: O is complete after it
                int kt;
                uint32_t u, ob, j;
            } pend{false, false, 0, 0, 0, 0};
            auto issue_pv = [&]() -> bool {
                if (!pend.live) return true;
                const uint32_t vb = pend.u & 1;
                // O buffer ob is free once item j - 2's epilogue has read it.
                if (pend.kt == 0 && !wait_bar(&bars->o_empty[pend.ob], ((pend.j >> 1) & 1u) ^ 1u, failed)) return false;
                if (!wait_bar(&bars->v_full[vb], (pend.u >> 1) & 1u, failed) || !wait_bar(&bars->p_full, pend.u & 1u, failed))
                    return false;
                fence_async_smem();
                fence_after();
                const uint32_t aV = smem_u32(sV0 + vb * kTileBytes);
                const uint32_t tO = tmem + kTmemO + pend.ob * 128u;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t blk = static_cast<uint32_t>(kk >> 2) * kBlkBytes;
                    const uint64_t step = 2ull * static_cast<uint64_t>(kk & 3);
                    // P (K-major A, 16 keys per step), V rows (MN-major B, 2 KB per 16 rows)
                    mma(tO, desc_kmajor(aP + blk) + step, desc_mnmajor(aV + static_cast<uint32_t>(kk) * 2048u),
                        idesc_pv<kF16>(), (pend.kt > 0 || kk > 0) ? 1 : 0);
                }
                commit(&bars->p_free);
                commit(&bars->v_empty[vb]);
                if (pend.last) commit(&bars->o_full[pend.ob]);
                pend.live = false;
                return true;
            };
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++j) {
                const ItemInfo f = item_info(p, it);
                if (!f.ok) break;                  // the loaders report it
                const uint32_t qb = j & 1;
                const uint32_t aQ = smem_u32(sQ0 + qb * kTileBytes);
                if (!wait_bar(&bars->q_full[qb], (j >> 1) & 1u, failed)) {
                    ok = false;
                    break;
                }
                for (int kt = 0; kt < f.n_kt; ++kt) {
                    const uint32_t kb = ku & 1, use = (ku >> 1) & 1u;
                    if (!wait_bar(&bars->k_full[kb], use, failed) || !wait_bar(&bars->s_free[kb], use ^ 1u, failed)) {
                        ok = false;
                        break;
                    }
                    fence_async_smem();     // loader-written tile -> async proxy (tcgen05.mma operand)
                    fence_after();
                    const uint32_t aK = smem_u32(sK0 + kb * kTileBytes);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t blk = static_cast<uint32_t>(kk >> 2) * kBlkBytes;
                        const uint64_t step = 2ull * static_cast<uint64_t>(kk & 3);
                        mma(tmem + kb * 128u, desc_kmajor(aQ + blk) + step, desc_kmajor(aK + blk) + step,
                            idesc_s<kF16>(), kk > 0);
                    }
                    any = true;
                    commit(&bars->s_full[kb]);
                    commit(&bars->k_empty[kb]);
                    if (kt == f.n_kt - 1) commit(&bars->q_empty[qb]);   // Q is read by S MMAs only
                    ++ku;
                    if (!issue_pv()) {
                        ok = false;
                        break;
                    }
                    pend = Pending{true, kt == f.n_kt - 1, kt, ku - 1, qb, j};
                }
            }
            if (ok && !issue_pv()) ok = false;
            if (!ok) {
                if (!*failed) report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, blockIdx.x, 1 << 21);
                *failed = 1;
            }
            // Every MMA this thread issued has completed before TMEM is freed (error path too).
            if (any) {
                commit(&bars->mma_done);
                mbar_wait(&bars->mma_done, 0, kWaitLimitCycles);
            }
        }
        __syncwarp();
    } else {
        // ============ softmax / epilogue: two warpgroups, thread = (query row, key half) ============
        const int sg = (warp - kSoftmaxWarp0) >> 2;       // columns [64 sg, 64 sg + 64) of S, P and O
        const int quad = warp & 3;
        const int r = 32 * quad + lane;          // TMEM lane and MMA row
        const int h = r >> 6, i = r & 63;
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * quad) << 16);
        uint32_t su = 0, xu = 0, j = 0;
        // Row hand-over with the other half: publish v, return the other half's value.
        auto exchange = [&](float v, float &other) -> bool {
            const uint32_t xs = xu & 1;
            xr[(xs * 2 + sg) * 128 + r] = v;
            mbar_arrive(&bars->x_ready[xs]);
            const bool ok = wait_bar(&bars->x_ready[xs], (xu >> 1) & 1u, failed);
            other = xr[(xs * 2 + (1 - sg)) * 128 + r];
            ++xu;
            return ok;
        };
        for (int it = blockIdx.x; it < n_items; it += gridDim.x, ++j) {
            const ItemInfo f = item_info(p, it);
            if (!f.ok) break;                      // the loaders report it
            const bool real = i < f.nq;
            const int pos_r = f.pos0 + (real ? i : f.nq - 1);
            const uint32_t ob = j & 1;
            const uint32_t tO = lane_addr + kTmemO + ob * 128u + static_cast<uint32_t>(64 * sg);
            // m_ref: the row's reference max (log2 domain) shared by both halves; l_run: this half's sum.
            float m_ref = -INFINITY, l_run = 0.0f;
            bool go = true;
            for (int kt = 0; kt < f.n_kt; ++kt) {
                const uint32_t sb = su & 1, par = (su >> 1) & 1u;
                // Every exit decision is warp-uniform: tcgen05.ld / st are .sync.aligned.
                go = wait_bar(&bars->s_full[sb], par, failed);
                if (!__all_sync(0xffffffffu, go)) break;
                fence_after();
                uint32_t sr[2][32];
                tmem_ld32_issue(lane_addr + sb * 128u + static_cast<uint32_t>(64 * sg), sr[0]);
                tmem_ld32_issue(lane_addr + sb * 128u + static_cast<uint32_t>(64 * sg + 32), sr[1]);
                tmem_wait_ld();
                // S buffer read out: the issuer may compute the next-but-one tile into it.
                fence_before();
                mbar_arrive(&bars->s_free[sb]);
                float sv[64];
                const int key0 = kt * kKeyTile + 64 * sg;
                float tm = -INFINITY;
#pragma unroll
                for (int jj = 0; jj < 64; ++jj) {
                    sv[jj] = key0 + jj > pos_r ? -INFINITY : __uint_as_float(sr[jj >> 5][jj & 31]);
                    tm = fmaxf(tm, sv[jj]);
                }
                // Tile max of the row over both halves.
                float tm_other;
                go = exchange(tm, tm_other);
                if (!__all_sync(0xffffffffu, go)) break;
                tm = fmaxf(tm, tm_other);
                // Key 0 is in tile 0 and never masked, so m_ref is finite from tile 0 on.
                float alpha = 1.0f;
                bool rescale = false;
                if (kt == 0) {
                    m_ref = tm;
                } else if (tm > m_ref + kRescaleLog2) {
                    alpha = ex2_approx(m_ref - tm);
                    m_ref = tm;
                    l_run *= alpha;
                    rescale = true;
                }
                uint32_t packed[32];
                float acc = 0.0f;
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    const float e0 = ex2_approx(sv[2 * jj] - m_ref), e1 = ex2_approx(sv[2 * jj + 1] - m_ref);
                    acc += e0 + e1;
                    packed[jj] = pack2<kF16>(e0, e1);
                }
                l_run += acc;
                // P V of the previous tile has completed: the P tile is free and O is at rest
                // (P V of this tile waits for P).
                go = wait_bar(&bars->p_free, (su & 1u) ^ 1u, failed);
                if (!__all_sync(0xffffffffu, go)) break;
                if (__any_sync(0xffffffffu, rescale)) {
                    fence_after();
#pragma unroll 1
                    for (int ch = 0; ch < 2; ++ch) {
                        float o[32];
                        tmem_ld32(tO + 32u * ch, o);
#pragma unroll
                        for (int c = 0; c < 32; ++c) o[c] *= alpha;
                        tmem_st32(tO + 32u * ch, o);
                    }
                    tmem_wait_st();
                }
                // keys 64 sg .. +63 = block sg of P (8 chunks of 8 keys)
                uint8_t *blk = sP + sg * kBlkBytes;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    *reinterpret_cast<uint4 *>(blk + swz(r, c)) =
                        make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
                }
                fence_async_smem();
                fence_before();
                mbar_arrive(&bars->p_full);
                ++su;
            }
            if (!__all_sync(0xffffffffu, go)) break;
            // Row sum over both halves.
            float l_other;
            go = exchange(l_run, l_other);
            if (!__all_sync(0xffffffffu, go)) break;
            const float inv_l = 1.0f / (l_run + l_other);
            // Epilogue: dims [64 sg, 64 sg + 64) of the O row -> attention output of (query i, head 2g+h)
            go = wait_bar(&bars->o_full[ob], (j >> 1) & 1u, failed);
            if (!__all_sync(0xffffffffu, go)) break;   // warp-uniform: the whole warp loads TMEM
            fence_after();
            const size_t off = static_cast<size_t>(f.row0 + (real ? i : 0)) * kQDim + (2 * f.g + h) * kHeadDim + 64 * sg;
#pragma unroll 1
            for (int ch = 0; ch < 2; ++ch) {
                float o[32];
                tmem_ld32(lane_addr + kTmemO + ob * 128u + static_cast<uint32_t>(64 * sg + 32 * ch), o);
                if (ch == 1) {
                    // O buffer ob read out: item j + 2 may accumulate into it.
                    fence_before();
                    mbar_arrive(&bars->o_empty[ob]);
                }
                if (!real) continue;
#pragma unroll
                for (int c = 0; c < 32; ++c) o[c] *= inv_l;
                if (p.out_bf16) {
                    __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(p.out) + off + ch * 32;
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        reinterpret_cast<uint4 *>(dst)[c] =
                            make_uint4(pack_bf16x2(o[8 * c], o[8 * c + 1]), pack_bf16x2(o[8 * c + 2], o[8 * c + 3]),
                                       pack_bf16x2(o[8 * c + 4], o[8 * c + 5]), pack_bf16x2(o[8 * c + 6], o[8 * c + 7]));
                } else {
                    float *dst = static_cast<float *>(p.out) + off + ch * 32;
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        reinterpret_cast<float4 *>(dst)[c] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                }
            }
        }
    }
    fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// Rows of q (f32) x scale rounded to the 16-bit operand type; 8 elements per thread.
__global__ void q_to16_kernel(const float *__restrict__ q, size_t n8, float scale, int f16, uint16_t *out) {
    pdl_trigger();
    pdl_wait();
    for (size_t t = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; t < n8;
         t += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float4 a = reinterpret_cast<const float4 *>(q)[2 * t];
        const float4 b = reinterpret_cast<const float4 *>(q)[2 * t + 1];
        const float s = scale;
        uint4 w;
        if (f16) w = make_uint4(pack_h2(a.x * s, a.y * s), pack_h2(a.z * s, a.w * s), pack_h2(b.x * s, b.y * s),
                                pack_h2(b.z * s, b.w * s));
        else w = make_uint4(pack_bf16x2(a.x * s, a.y * s), pack_bf16x2(a.z * s, a.w * s),
                            pack_bf16x2(b.x * s, b.y * s), pack_bf16x2(b.z * s, b.w * s));
        reinterpret_cast<uint4 *>(out)[t] = w;
    }
}

// Dynamic shared memory of a K3 launch: the layout plus room to reach a
// 1024-byte boundary, capped at the device's per-block maximum (the kernel
// checks that its layout fits what it was given).
cudaError_t k3_smem_bytes(size_t *bytes) {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    const size_t want = kSmemNeed + 1023;
    *bytes = want < static_cast<size_t>(optin) ? want : static_cast<size_t>(optin);
    return cudaSuccess;
}

}  // namespace

cudaError_t prepare_prefill_tc() {
    size_t smem = 0;
    cudaError_t e = k3_smem_bytes(&smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(prefill_attn_tc_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(prefill_attn_tc_kernel<uint8_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem));
}

bool prefill_tc_supported(int kv_dtype) { return kv_dtype == kKvBF16 || kv_is_8bit(kv_dtype); }

cudaError_t launch_q_to16(const float *q, int n, float scale, bool f16, void *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const size_t n8 = static_cast<size_t>(n) * kQDim / 8;
    const size_t blocks = (n8 + 255) / 256;
    return launch_pdl(q_to16_kernel, dim3(static_cast<unsigned>(blocks < 4096 ? blocks : 4096)), dim3(256), 0, st, q,
                      n8, scale, f16 ? 1 : 0, static_cast<uint16_t *>(out));
}

cudaError_t launch_prefill_attn_tc(const PrefillAttnParams &pp, int kv_dtype, const int4 *items, int n_items,
                                   bool out_bf16, cudaStream_t st) {
    if (n_items <= 0) return cudaSuccess;
    if (!prefill_tc_supported(kv_dtype) || (kv_is_8bit(kv_dtype) && !pp.scales) || !pp.q16) return cudaErrorInvalidValue;
    K3Params p{};
    p.items = items;
    p.slots = pp.slots;
    p.positions = pp.positions;
    p.q16 = static_cast<const uint16_t *>(pp.q16);
    p.out = pp.out;
    p.out_bf16 = out_bf16 ? 1 : 0;
    p.pool = pp.pool;
    p.scales = pp.scales;
    p.page_table = pp.page_table;
    p.maxp = pp.maxp;
    p.max_streams = pp.max_streams;
    p.n_pages = pp.n_pages;
    p.err = pp.err;
    p.v_int8 = kv_dtype == kKvE4I8 ? 1 : 0;
    int dev = 0, sms = 0;
    size_t smem = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = k3_smem_bytes(&smem);
    if (e != cudaSuccess) return e;
    const int grid = n_items < sms ? n_items : sms;   // persistent: one CTA per SM walks the items
    if (kv_dtype == kKvBF16)
        return launch_pdl(prefill_attn_tc_kernel<__nv_bfloat16>, dim3(grid), dim3(kThreads), smem, st, p, n_items);
    return launch_pdl(prefill_attn_tc_kernel<uint8_t>, dim3(grid), dim3(kThreads), smem, st, p, n_items);
}

}  // namespace qkv
