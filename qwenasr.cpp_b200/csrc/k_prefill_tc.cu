// K3: causal prefill attention on the tensor cores (tcgen05 + TMEM), bf16 cache.
// Replaces the prompt half of text-decoder.cpp:322-334 (QK^T, diag mask,
// softmax, PV over the whole prompt) for the paged cache that K1 has just
// filled (and the scalar twin :739-791).
//
// One CTA per work item = (64 consecutive queries of one stream, kv head g).
// GQA: the two q heads of kv head g share the item, so the MMA's M = 128 rows
// are [64 queries of head 2g | 64 queries of head 2g+1] and every K/V tile is
// fetched once for both.  Keys come in tiles of 128 (8 pages): a tensor map
// over the pool ([pool rows][128] bf16, box 16 rows x 64 columns, 128-byte
// swizzle) brings each page's K or V rows straight into the canonical UMMA
// layouts — K as the K-major B operand of S = Q K^T, V as the MN-major B
// operand of O += P V.
//
// Two passes over the key tiles: pass 1 computes each row's running max and
// sum from S (TMEM -> registers); pass 2 recomputes S, writes the normalised
// P (bf16, swizzled) to shared memory and accumulates O = P V in TMEM, so O
// never needs rescaling.  Roles: warp 0 TMA producer, warp 1 TMEM allocator +
// MMA issuer, warps 2..5 = 128 softmax/epilogue threads (thread = TMEM lane =
// one query row).  All waits bounded.
#include "kernels.h"

#include <cuda.h>

namespace qkv {

bool tc_tensor_map(CUtensorMap *out, const void *ptr, int rows, int K, int box_rows);

namespace {

constexpr int kQPerItem = 64;
constexpr int kKeyTile = 128;
constexpr int kPagesPerTile = kKeyTile / kPageTokens;     // 8
constexpr uint32_t kBlkBytes = 128 * 128;                 // [128 rows][64 bf16], 16 KB
constexpr uint32_t kTileBytes = 2 * kBlkBytes;            // two 64-column blocks, 32 KB
constexpr int kThreads = 192;
constexpr size_t kSmem = 1024 + 4 * static_cast<size_t>(kTileBytes) + 256;
constexpr uint32_t kTmemCols = 256;                       // S: cols [0,128), O: cols [128,256)

struct K3Params {
    const int4 *items;      // (row0, nq, g, 0)
    const int *slots;
    const int *positions;
    const float *q;         // [rows][2048] post-RoPE
    void *out;              // [rows][2048]
    int out_bf16;
    const int *page_table;
    int maxp;
    int max_streams;
    int n_pages;
    float scale_log2;
    DevError *err;
};

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Swizzled (128 B) operand descriptors, sm_100 version bit set.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t addr) {
    return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | ((1024ull >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// MN-major tile: 64-element MN blocks kBlkBytes apart (LBO), 8-row K groups 1024 B apart (SBO).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t addr) {
    return ((addr >> 4) & 0x3FFFull) | (static_cast<uint64_t>(kBlkBytes >> 4) << 16) | ((1024ull >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}

constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescPV = kIdescS | (1u << 16);   // B (V) MN-major

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

struct Bars {
    uint64_t q_ready, k_full, k_empty, v_full, v_empty, s_full, s_free, p_full, p_free, o_done;
};

__global__ void __launch_bounds__(kThreads, 1)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap pool_map, K3Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem, *sK = smem + kTileBytes, *sV = smem + 2 * kTileBytes, *sP = smem + 3 * kTileBytes;
    Bars *bars = reinterpret_cast<Bars *>(smem + 4 * kTileBytes);
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
    const bool item_ok = slot >= 0 && slot < p.max_streams && pos0 >= 0 && nq > 0 && key_pages <= p.maxp;

    if (threadIdx.x == 0) {
        mbar_init(&bars->q_ready, 128);
        mbar_init(&bars->k_full, 1);
        mbar_init(&bars->k_empty, 1);
        mbar_init(&bars->v_full, 1);
        mbar_init(&bars->v_empty, 1);
        mbar_init(&bars->s_full, 1);
        mbar_init(&bars->s_free, 128);
        mbar_init(&bars->p_full, 128);
        mbar_init(&bars->p_free, 1);
        mbar_init(&bars->o_done, 1);
        *failed = item_ok ? 0 : 1;
        if (!item_ok) report_error(p.err, kErrRowBounds, kWherePrefillAttn, row0, pos0);
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_uses = *failed ? 0 : 2 * n_kt;

    if (warp == 0) {
        // ================= TMA producer =================
        if (lane == 0 && n_uses > 0) {
            const int *pt = p.page_table + static_cast<size_t>(slot) * p.maxp;
            int k_issued = 0, v_issued = 0;
            for (int u = 0; u < n_uses && !*failed; ++u) {
                const int pass = u / n_kt, kt = u % n_kt;
                int pages[kPagesPerTile];
                bool bad = false;
                for (int j = 0; j < kPagesPerTile; ++j) {
                    const int pi = kt * kPagesPerTile + j;
                    // Key slots past the stream's last page reuse its first page: finite
                    // values, masked out of S, multiplied by P = 0 in P V.
                    int pg = pt[pi < key_pages ? pi : 0];
                    if (pg < 0 || pg >= p.n_pages) bad = true;
                    pages[j] = pg;
                }
                if (bad) {
                    report_error(p.err, kErrPageIndex, kWherePrefillAttn, row0, kt);
                    *failed = 1;
                    break;
                }
                if (!mbar_wait(&bars->k_empty, (static_cast<uint32_t>(u) & 1u) ^ 1u, kWaitLimitCycles)) {
                    report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, row0, u);
                    *failed = 1;
                    break;
                }
                mbar_arrive_expect_tx(&bars->k_full, kTileBytes);
                for (int j = 0; j < kPagesPerTile; ++j) {
                    const int krow = ((pages[j] * 2 + 0) * kHkv + g) * kPageTokens;
                    tma_load_2d(sK + j * 2048, &pool_map, 0, krow, &bars->k_full);
                    tma_load_2d(sK + kBlkBytes + j * 2048, &pool_map, 64, krow, &bars->k_full);
                }
                ++k_issued;
                if (pass == 1) {
                    if (!mbar_wait(&bars->v_empty, (static_cast<uint32_t>(kt) & 1u) ^ 1u, kWaitLimitCycles)) {
                        report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, row0, -u);
                        *failed = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&bars->v_full, kTileBytes);
                    for (int j = 0; j < kPagesPerTile; ++j) {
                        const int vrow = ((pages[j] * 2 + 1) * kHkv + g) * kPageTokens;
                        tma_load_2d(sV + j * 2048, &pool_map, 0, vrow, &bars->v_full);
                        tma_load_2d(sV + kBlkBytes + j * 2048, &pool_map, 64, vrow, &bars->v_full);
                    }
                    ++v_issued;
                }
            }
            // Drain the last loads of each buffer before the CTA may exit.
            if (k_issued > 0) mbar_wait(&bars->k_full, static_cast<uint32_t>(k_issued - 1) & 1u, kWaitLimitCycles);
            if (v_issued > 0) mbar_wait(&bars->v_full, static_cast<uint32_t>(v_issued - 1) & 1u, kWaitLimitCycles);
        }
    } else if (warp == 1) {
        // ================= MMA issuer =================
        if (lane == 0) {
            int issued = 0;
            bool ok = n_uses > 0 && mbar_wait(&bars->q_ready, 0, kWaitLimitCycles);
            if (n_uses > 0 && !ok) {
                report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, row0, 1 << 20);
                *failed = 1;
            }
            const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP);
            for (int u = 0; ok && u < n_uses; ++u) {
                const int pass = u / n_kt, kt = u % n_kt;
                if (!mbar_wait(&bars->k_full, static_cast<uint32_t>(u) & 1u, kWaitLimitCycles) ||
                    (u > 0 && !mbar_wait(&bars->s_free, static_cast<uint32_t>(u - 1) & 1u, kWaitLimitCycles))) {
                    ok = false;
                    break;
                }
                fence_after();
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t blk = static_cast<uint32_t>(kk >> 2) * kBlkBytes;
                    const uint64_t step = 2ull * static_cast<uint64_t>(kk & 3);
                    mma(tmem, desc_kmajor(aQ + blk) + step, desc_kmajor(aK + blk) + step, kIdescS, kk > 0);
                }
                ++issued;
                commit(&bars->s_full);
                commit(&bars->k_empty);
                if (pass == 1) {
                    if (!mbar_wait(&bars->v_full, static_cast<uint32_t>(kt) & 1u, kWaitLimitCycles) ||
                        !mbar_wait(&bars->p_full, static_cast<uint32_t>(kt) & 1u, kWaitLimitCycles)) {
                        ok = false;
                        break;
                    }
                    fence_after();
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t blk = static_cast<uint32_t>(kk >> 2) * kBlkBytes;
                        const uint64_t step = 2ull * static_cast<uint64_t>(kk & 3);
                        // 16 keys per step: P columns (K-major), V rows (MN-major, 2 KB per 16 rows)
                        mma(tmem + 128, desc_kmajor(aP + blk) + step, desc_mnmajor(aV + static_cast<uint32_t>(kk) * 2048u),
                            kIdescPV, (kt > 0 || kk > 0) ? 1 : 0);
                    }
                    commit(&bars->p_free);
                    commit(&bars->v_empty);
                }
            }
            if (!ok && n_uses > 0) {
                report_error(p.err, kErrWaitTimeout, kWherePrefillAttn, row0, 1 << 21);
                *failed = 1;
            }
            // o_done completes when every issued MMA has, on the error path too.
            if (issued > 0) commit(&bars->o_done);
            else mbar_arrive(&bars->o_done);
            mbar_wait(&bars->o_done, 0, kWaitLimitCycles);
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
            // Q row (scaled into the log2 domain, bf16, swizzled K-major)
            const float *qrow = p.q + static_cast<size_t>(row0 + (real ? i : 0)) * kQDim + (2 * g + h) * kHeadDim;
#pragma unroll 1
            for (int c16 = 0; c16 < 16; ++c16) {
                uint4 w = make_uint4(0, 0, 0, 0);
                if (real) {
                    const float4 a = reinterpret_cast<const float4 *>(qrow + c16 * 8)[0];
                    const float4 b = reinterpret_cast<const float4 *>(qrow + c16 * 8)[1];
                    const float s = p.scale_log2;
                    w.x = pack_bf16x2(a.x * s, a.y * s);
                    w.y = pack_bf16x2(a.z * s, a.w * s);
                    w.z = pack_bf16x2(b.x * s, b.y * s);
                    w.w = pack_bf16x2(b.z * s, b.w * s);
                }
                *reinterpret_cast<uint4 *>(sQ + (c16 >> 3) * kBlkBytes + swz(r, c16 & 7)) = w;
            }
            fence_async_smem();
            mbar_arrive(&bars->q_ready);
        }
        float m_run = -INFINITY, l_run = 0.0f, inv_l = 0.0f;
        for (int u = 0; u < n_uses; ++u) {
            const int pass = u / n_kt, kt = u % n_kt;
            // Every exit decision is warp-uniform: the tcgen05.ld below is .sync.aligned.
            bool go = !*failed && mbar_wait(&bars->s_full, static_cast<uint32_t>(u) & 1u, kWaitLimitCycles);
            if (!__all_sync(0xffffffffu, go)) break;
            fence_after();
            if (pass == 1 && kt == 0) inv_l = 1.0f / l_run;
            if (pass == 1 && kt > 0) {
                go = mbar_wait(&bars->p_free, static_cast<uint32_t>(kt - 1) & 1u, kWaitLimitCycles);
                if (!__all_sync(0xffffffffu, go)) break;
            }
#pragma unroll 1
            for (int ch = 0; ch < 4; ++ch) {
                float s[32];
                tmem_ld32(lane_addr + static_cast<uint32_t>(ch * 32), s);
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
                    uint32_t packed[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        packed[j] = pack_bf16x2(exp2f(s[2 * j] - m_run) * inv_l, exp2f(s[2 * j + 1] - m_run) * inv_l);
                    // keys ch*32 .. +31 = 4 chunks of 8 in block ch >> 1
                    uint8_t *blk = sP + (ch >> 1) * kBlkBytes;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int chunk = (ch & 1) * 4 + c;
                        *reinterpret_cast<uint4 *>(blk + swz(r, chunk)) =
                            make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
                    }
                }
            }
            fence_before();
            mbar_arrive(&bars->s_free);
            if (pass == 1) {
                fence_async_smem();
                mbar_arrive(&bars->p_full);
            }
        }
        // Epilogue: O row (128 dims) -> attention output of (query i, head 2g+h)
        bool done = n_uses > 0 && mbar_wait(&bars->o_done, 0, kWaitLimitCycles) && !*failed;
        done = __all_sync(0xffffffffu, done);   // warp-uniform: the whole warp loads TMEM, only real rows store
        fence_after();
        if (done) {
            const size_t off = static_cast<size_t>(row0 + (real ? i : 0)) * kQDim + (2 * g + h) * kHeadDim;
#pragma unroll 1
            for (int ch = 0; ch < 4; ++ch) {
                float o[32];
                tmem_ld32(lane_addr + 128u + static_cast<uint32_t>(ch * 32), o);
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
    if (warp == 1) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

}  // namespace

cudaError_t prepare_prefill_tc() {
    return cudaFuncSetAttribute(prefill_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kSmem));
}

cudaError_t launch_prefill_attn_tc(const PrefillAttnParams &pp, const int4 *items, int n_items, bool out_bf16,
                                   cudaStream_t st) {
    if (n_items <= 0) return cudaSuccess;
    CUtensorMap map;
    const long long rows = static_cast<long long>(pp.n_pages) * 2 * kHkv * kPageTokens;
    if (rows > 0x7fffffffLL || !tc_tensor_map(&map, pp.pool, static_cast<int>(rows), kHeadDim, kPageTokens))
        return cudaErrorInvalidValue;
    K3Params p{};
    p.items = items;
    p.slots = pp.slots;
    p.positions = pp.positions;
    p.q = pp.q;
    p.out = pp.out;
    p.out_bf16 = out_bf16 ? 1 : 0;
    p.page_table = pp.page_table;
    p.maxp = pp.maxp;
    p.max_streams = pp.max_streams;
    p.n_pages = pp.n_pages;
    p.scale_log2 = pp.scale_log2;
    p.err = pp.err;
    prefill_attn_tc_kernel<<<n_items, kThreads, kSmem, st>>>(map, p);
    return cudaGetLastError();
}

}  // namespace qkv
