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
// Operand staging: a warpgroup of 128 loader threads, one key row each, reads
// the row straight from its page with 16-byte loads and writes it into the
// canonical 128-byte-swizzled UMMA layout — K as the K-major B operand of
// S = Q K^T, V as the MN-major B operand of O += P V.  (A page contributes
// 16 scattered rows per head; one TMA copy per page and column block would be
// bounded by the rate at which a thread can issue copies.)  For the e4m3 cache
// the loader dequantises on the way (e4m3 -> f16 exactly, times the page's
// per-(kv, head) scale in f16), and Q, P are f16 too; for bf16 everything is
// bf16.  K and V tiles are double-buffered, S is double-buffered in TMEM.
//
// Two passes over the key tiles: pass 1 computes each row's running max and
// sum from S (TMEM -> registers); pass 2 recomputes S, writes the normalised
// P (swizzled) to shared memory and accumulates O = P V in TMEM, so O never
// needs rescaling.  In pass 2 the issuer puts S of tile t ahead of P V of
// tile t-1, so the softmax of t overlaps the PV MMAs of t-1.
//
// Roles: warps 0..3 loaders, warps 4..7 softmax/epilogue (thread = TMEM lane
// = one query row; lane quadrant = warp % 4), warp 8 TMEM allocator + MMA
// issuer (one thread).  All waits bounded.
#include "kernels.h"

namespace qkv {

namespace {

constexpr int kQPerItem = 64;
constexpr int kKeyTile = 128;
constexpr uint32_t kBlkBytes = 128 * 128;                 // [128 rows][64 x 16-bit], 16 KB
constexpr uint32_t kTileBytes = 2 * kBlkBytes;            // two 64-column blocks, 32 KB
constexpr int kMmaWarp = 8;
constexpr int kThreads = 9 * 32;
// Q, K[2], V[2], P tiles + barriers
constexpr size_t kSmem = 1024 + 6 * static_cast<size_t>(kTileBytes) + 512;
constexpr uint32_t kTmemCols = 512;                       // S0 [0,128), S1 [128,256), O [256,384)
constexpr uint32_t kTmemO = 256;

struct K3Params {
    const int4 *items;      // (row0, nq, g, 0)
    const int *slots;
    const int *positions;
    const float *q;         // [rows][2048] post-RoPE
    void *out;              // [rows][2048]
    int out_bf16;
    const void *pool;
    const float *scales;    // e4m3 cache: [pages][2][8]
    const int *page_table;
    int maxp;
    int max_streams;
    int n_pages;
    float scale_log2;
    DevError *err;
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

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
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

// One key row (128 dims of page `page`, kv half `kv`, head g, token `tok`) in
// registers: 16 x 16 B of bf16, or 8 x 16 B of e4m3 (+ its page scale).  A key
// past the stream's length (`live` false) is not read and stores as zeros.
template <typename TC> struct RowRegs {
    static constexpr int kWords = sizeof(TC) == 2 ? 16 : 8;
    uint4 w[kWords];
    float scale;
    bool live;
};

template <typename TC>
__device__ __forceinline__ void fetch_row(const K3Params &p, RowRegs<TC> &rr, int page, int kv, int g, int tok,
                                          bool live) {
    rr.live = live;
    rr.scale = 1.0f;
    if (!live) return;
    const size_t row = ((static_cast<size_t>(page) * 2 + kv) * kHkv + g) * kPageTokens + tok;
    const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(p.pool) + row * kHeadDim * sizeof(TC));
#pragma unroll
    for (int c = 0; c < RowRegs<TC>::kWords; ++c) rr.w[c] = __ldg(src + c);
    if constexpr (sizeof(TC) == 1) rr.scale = __ldg(p.scales + (static_cast<size_t>(page) * 2 + kv) * kHkv + g);
}

// Row r of a swizzled [2 blocks][128 rows][64] 16-bit tile (e4m3: dequantised
// exactly to f16, then times the page scale in f16).
template <typename TC>
__device__ __forceinline__ void store_row(uint8_t *tile, int r, const RowRegs<TC> &rr) {
    if (!rr.live) {
#pragma unroll
        for (int c = 0; c < 16; ++c)
            *reinterpret_cast<uint4 *>(tile + (c >> 3) * kBlkBytes + swz(r, c & 7)) = make_uint4(0, 0, 0, 0);
        return;
    }
    if constexpr (sizeof(TC) == 2) {
#pragma unroll
        for (int c = 0; c < 16; ++c) *reinterpret_cast<uint4 *>(tile + (c >> 3) * kBlkBytes + swz(r, c & 7)) = rr.w[c];
    } else {
        const uint32_t s2 = pack_h2(rr.scale, rr.scale);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            // 16 e4m3 = dims 16c .. 16c+15 -> f16 chunks 2c (dims 16c..+7) and 2c+1
            const uint32_t ws[4] = {rr.w[c].x, rr.w[c].y, rr.w[c].z, rr.w[c].w};
            uint32_t h[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                uint32_t lo2, hi2;
                e4m3x4_to_h2x2(ws[k], lo2, hi2);
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
    uint64_t q_ready, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], s_free[2], p_full, p_free, o_done;
};

__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity) {
    return mbar_wait(bar, parity, kWaitLimitCycles);
}

template <typename TC>
__global__ void __launch_bounds__(kThreads, 1) prefill_attn_tc_kernel(K3Params p) {
    constexpr bool kF16 = sizeof(TC) == 1;   // e4m3 cache -> f16 operands
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem;
    uint8_t *const sK0 = smem + kTileBytes;         // K[b] = sK0 + b * kTileBytes
    uint8_t *const sV0 = smem + 3 * kTileBytes;     // V[b] = sV0 + b * kTileBytes
    uint8_t *sP = smem + 5 * kTileBytes;
    Bars *bars = reinterpret_cast<Bars *>(smem + 6 * kTileBytes);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 1);
    volatile int *failed = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int4 item = p.items[blockIdx.x];
    const int row0 = item.x, nq = item.y, g = item.z;
    const int slot = p.slots[row0];
    const int pos0 = p.positions[row0];
    const int kv_len = pos0 + nq;
    const int n_kt = (kv_len + kKeyTile - 1) / kKeyTile;
    const int key_pages = (kv_len + kPageTokens - 1) / kPageTokens;
    const bool item_ok = slot >= 0 && slot < p.max_streams && pos0 >= 0 && nq > 0 && nq <= kQPerItem &&
                         key_pages <= p.maxp && g >= 0 && g < kHkv;
    const int *pt = p.page_table + static_cast<size_t>(item_ok ? slot : 0) * p.maxp;

    if (threadIdx.x == 0) {
        mbar_init(&bars->q_ready, 128);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->k_full[b], 128);
            mbar_init(&bars->k_empty[b], 1);
            mbar_init(&bars->v_full[b], 128);
            mbar_init(&bars->v_empty[b], 1);
            mbar_init(&bars->s_full[b], 1);
            mbar_init(&bars->s_free[b], 128);
        }
        mbar_init(&bars->p_full, 128);
        mbar_init(&bars->p_free, 1);
        mbar_init(&bars->o_done, 1);
        *failed = item_ok ? 0 : 1;
        if (!item_ok) report_error(p.err, kErrRowBounds, kWherePrefillAttn, row0, pos0);
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
    // Every page id of the item's keys, checked once by the whole CTA.
    if (item_ok) {
        for (int i = threadIdx.x; i < key_pages; i += kThreads) {
            const int pg = pt[i];
            if (pg < 0 || pg >= p.n_pages) {
                report_error(p.err, kErrPageIndex, kWherePrefillAttn, row0, i);
                *failed = 1;
            }
        }
    }
    __syncthreads();
    const uint32_t tmem = *tmem_slot;
    const int n_uses = *failed ? 0 : 2 * n_kt;

    if (warp < 4) {
        // ================= loaders: thread = key row of the tile =================
        const int r = threadIdx.x;
        for (int u = 0; u < n_uses; ++u) {
            const int pass = u / n_kt, kt = u % n_kt;
            const int key = kt * kKeyTile + r;
            // Keys past the stream's length are zero rows (masked out of S,
            // multiplied by P = 0 in P V); their page index is clamped.
            const int pi = key / kPageTokens;
            const int page = pt[pi < key_pages ? pi : 0];
            const int tok = key % kPageTokens;
            const int kb = u & 1;
            // K (and, in pass 2, V) loads in flight together before either buffer is waited on.
            RowRegs<TC> kr, vr;
            fetch_row<TC>(p, kr, page, 0, g, tok, key < kv_len);
            if (pass == 1) fetch_row<TC>(p, vr, page, 1, g, tok, key < kv_len);
            if (*failed || !wait_bar(&bars->k_empty[kb], ((static_cast<uint32_t>(u) >> 1) & 1u) ^ 1u)) {
                if (!*failed) report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, row0, u);
                *failed = 1;
                break;
            }
            store_row<TC>(sK0 + kb * kTileBytes, r, kr);
            fence_async_smem();
            mbar_arrive(&bars->k_full[kb]);
            if (pass == 1) {
                const int vb = kt & 1;
                if (*failed || !wait_bar(&bars->v_empty[vb], ((static_cast<uint32_t>(kt) >> 1) & 1u) ^ 1u)) {
                    if (!*failed) report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, row0, -u);
                    *failed = 1;
                    break;
                }
                store_row<TC>(sV0 + vb * kTileBytes, r, vr);
                fence_async_smem();
                mbar_arrive(&bars->v_full[vb]);
            }
        }
    } else if (warp == kMmaWarp) {
        // ================= MMA issuer =================
        if (lane == 0) {
            int issued = 0;
            bool ok = n_uses > 0 && wait_bar(&bars->q_ready, 0);
            if (n_uses > 0 && !ok) {
                report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, row0, 1 << 20);
                *failed = 1;
            }
            const uint32_t aQ = smem_u32(sQ), aP = smem_u32(sP);
            // P V of tile kt: P (K-major A, 16 keys per step), V rows (MN-major B, 2 KB per 16 rows).
            auto issue_pv = [&](int kt) -> bool {
                const int vb = kt & 1;
                if (*failed || !wait_bar(&bars->v_full[vb], (static_cast<uint32_t>(kt) >> 1) & 1u) ||
                    !wait_bar(&bars->p_full, static_cast<uint32_t>(kt) & 1u))
                    return false;
                fence_after();
                const uint32_t aV = smem_u32(sV0 + vb * kTileBytes);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t blk = static_cast<uint32_t>(kk >> 2) * kBlkBytes;
                    const uint64_t step = 2ull * static_cast<uint64_t>(kk & 3);
                    mma(tmem + kTmemO, desc_kmajor(aP + blk) + step, desc_mnmajor(aV + static_cast<uint32_t>(kk) * 2048u),
                        idesc_pv<kF16>(), (kt > 0 || kk > 0) ? 1 : 0);
                }
                ++issued;
                commit(&bars->p_free);
                commit(&bars->v_empty[vb]);
                return true;
            };
            for (int u = 0; ok && u < n_uses; ++u) {
                const int pass = u / n_kt, kt = u % n_kt;
                const int kb = u & 1, sb = u & 1;
                const uint32_t use = (static_cast<uint32_t>(u) >> 1) & 1u;
                if (*failed || !wait_bar(&bars->k_full[kb], use) || !wait_bar(&bars->s_free[sb], use ^ 1u)) {
                    ok = false;
                    break;
                }
                fence_after();
                const uint32_t aK = smem_u32(sK0 + kb * kTileBytes);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t blk = static_cast<uint32_t>(kk >> 2) * kBlkBytes;
                    const uint64_t step = 2ull * static_cast<uint64_t>(kk & 3);
                    mma(tmem + static_cast<uint32_t>(sb * 128), desc_kmajor(aQ + blk) + step,
                        desc_kmajor(aK + blk) + step, idesc_s<kF16>(), kk > 0);
                }
                ++issued;
                commit(&bars->s_full[sb]);
                commit(&bars->k_empty[kb]);
                if (pass == 1 && kt > 0 && !issue_pv(kt - 1)) {
                    ok = false;
                    break;
                }
            }
            if (ok && n_uses > 0 && !issue_pv(n_kt - 1)) ok = false;
            if (!ok && n_uses > 0) {
                report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, row0, 1 << 21);
                *failed = 1;
            }
            // o_done completes when every issued MMA has, on the error path too.
            if (issued > 0) commit(&bars->o_done);
            else mbar_arrive(&bars->o_done);
            wait_bar(&bars->o_done, 0);
        }
        __syncwarp();
    } else {
        // ================= softmax / epilogue: thread = query row =================
        const int quad = warp & 3;
        const int r = 32 * quad + lane;          // TMEM lane and MMA row
        const int h = r >> 6, i = r & 63;
        const bool real = i < nq;
        const int pos_r = pos0 + (real ? i : nq - 1);
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * quad) << 16);
        if (n_uses > 0) {
            // Q row, scaled into the log2 domain, swizzled K-major
            const float4 *qrow = reinterpret_cast<const float4 *>(
                p.q + static_cast<size_t>(row0 + (real ? i : 0)) * kQDim + (2 * g + h) * kHeadDim);
            const float s = p.scale_log2;
#pragma unroll
            for (int half_q = 0; half_q < 2; ++half_q) {
                // 64 dims per half: all 16 loads in flight before any is used
                float4 a[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) a[k] = real ? __ldg(qrow + half_q * 16 + k) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const float4 x = a[2 * c], y = a[2 * c + 1];
                    const uint4 w = make_uint4(pack2<kF16>(x.x * s, x.y * s), pack2<kF16>(x.z * s, x.w * s),
                                               pack2<kF16>(y.x * s, y.y * s), pack2<kF16>(y.z * s, y.w * s));
                    *reinterpret_cast<uint4 *>(sQ + half_q * kBlkBytes + swz(r, c)) = w;
                }
            }
            fence_async_smem();
            mbar_arrive(&bars->q_ready);
        }
        float m_run = -INFINITY, l_run = 0.0f, inv_l = 0.0f;
        for (int u = 0; u < n_uses; ++u) {
            const int pass = u / n_kt, kt = u % n_kt;
            const int sb = u & 1;
            // Every exit decision is warp-uniform: the tcgen05.ld below is .sync.aligned.
            bool go = !*failed && wait_bar(&bars->s_full[sb], (static_cast<uint32_t>(u) >> 1) & 1u);
            if (!__all_sync(0xffffffffu, go)) break;
            fence_after();
            if (pass == 1 && kt == 0) inv_l = 1.0f / l_run;
            uint32_t packed[4][16];
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                float s[32];
                tmem_ld32(lane_addr + static_cast<uint32_t>(sb * 128 + ch * 32), s);
                const int key0 = kt * kKeyTile + ch * 32;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (key0 + j > pos_r) s[j] = -INFINITY;
                }
                if (pass == 0) {
                    float cm = s[0];
#pragma unroll
                    for (int j = 1; j < 32; ++j) cm = fmaxf(cm, s[j]);
                    const float m_new = fmaxf(m_run, cm);
                    if (m_new != -INFINITY) {
                        float acc = 0.0f;
#pragma unroll
                        for (int j = 0; j < 32; ++j) acc += exp2f(s[j] - m_new);
                        l_run = l_run * exp2f(m_run - m_new) + acc;
                        m_run = m_new;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        packed[ch][j] = pack2<kF16>(exp2f(s[2 * j] - m_run) * inv_l, exp2f(s[2 * j + 1] - m_run) * inv_l);
                }
            }
            // S buffer sb read out: the issuer may compute the next-but-one tile into it.
            fence_before();
            mbar_arrive(&bars->s_free[sb]);
            if (pass == 1) {
                go = !*failed && wait_bar(&bars->p_free, (static_cast<uint32_t>(kt) & 1u) ^ 1u);
                if (!__all_sync(0xffffffffu, go)) break;
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) {
                    // keys ch*32 .. +31 = 4 chunks of 8 in block ch >> 1
                    uint8_t *blk = sP + (ch >> 1) * kBlkBytes;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int chunk = (ch & 1) * 4 + c;
                        *reinterpret_cast<uint4 *>(blk + swz(r, chunk)) =
                            make_uint4(packed[ch][4 * c], packed[ch][4 * c + 1], packed[ch][4 * c + 2], packed[ch][4 * c + 3]);
                    }
                }
                fence_async_smem();
                mbar_arrive(&bars->p_full);
            }
        }
        // Epilogue: O row (128 dims) -> attention output of (query i, head 2g+h)
        bool done = n_uses > 0 && wait_bar(&bars->o_done, 0) && !*failed;
        done = __all_sync(0xffffffffu, done);   // warp-uniform: the whole warp loads TMEM, only real rows store
        fence_after();
        if (done) {
            const size_t off = static_cast<size_t>(row0 + (real ? i : 0)) * kQDim + (2 * g + h) * kHeadDim;
#pragma unroll 1
            for (int ch = 0; ch < 4; ++ch) {
                float o[32];
                tmem_ld32(lane_addr + kTmemO + static_cast<uint32_t>(ch * 32), o);
                if (!real) continue;
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

}  // namespace

cudaError_t prepare_prefill_tc() {
    cudaError_t e = cudaFuncSetAttribute(prefill_attn_tc_kernel<__nv_bfloat16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmem));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(prefill_attn_tc_kernel<uint8_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kSmem));
}

bool prefill_tc_supported(int kv_dtype) { return kv_dtype == kKvBF16 || kv_dtype == kKvFP8; }

cudaError_t launch_prefill_attn_tc(const PrefillAttnParams &pp, int kv_dtype, const int4 *items, int n_items,
                                   bool out_bf16, cudaStream_t st) {
    if (n_items <= 0) return cudaSuccess;
    if (!prefill_tc_supported(kv_dtype) || (kv_dtype == kKvFP8 && !pp.scales)) return cudaErrorInvalidValue;
    K3Params p{};
    p.items = items;
    p.slots = pp.slots;
    p.positions = pp.positions;
    p.q = pp.q;
    p.out = pp.out;
    p.out_bf16 = out_bf16 ? 1 : 0;
    p.pool = pp.pool;
    p.scales = pp.scales;
    p.page_table = pp.page_table;
    p.maxp = pp.maxp;
    p.max_streams = pp.max_streams;
    p.n_pages = pp.n_pages;
    p.scale_log2 = pp.scale_log2;
    p.err = pp.err;
    if (kv_dtype == kKvBF16) prefill_attn_tc_kernel<__nv_bfloat16><<<n_items, kThreads, kSmem, st>>>(p);
    else prefill_attn_tc_kernel<uint8_t><<<n_items, kThreads, kSmem, st>>>(p);
    return cudaGetLastError();
}

}  // namespace qkv
