// Tensor-core projections on sm_100a: C[M][N] (+)= X[M][K] . W[N][K]^T with
// bf16 X and W, f32 accumulation in TMEM (tcgen05.mma kind::f16), operands
// staged by TMA (cp.async.bulk.tensor, 128-byte swizzle, no multicast).
// Replaces the reference's projections (text-decoder.cpp:371-373, 465, 469-472,
// 476-493: GGML mul_mat with GGML_PREC_F32).
//
// Swap-AB: the MMA's M side is 128 weight rows (output features) and its N
// side is a tile of BN tokens, so a decode step's handful of tokens is a
// legal N (16..256) while the weights stream through at full width.  Skinny
// shapes split K across CTAs (grid.z) and accumulate with f32 red.add, so a
// 1024-wide projection still puts ~150-300 CTAs on the memory system.
//
// CTA = 6 warps: warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer
// (one thread), warps 2..5 epilogue (TMEM lane quadrant = warp % 4, one
// weight row per thread).  Every mbarrier wait is bounded.
#include "kernels.h"

#include <cuda.h>

#include <mutex>
#include <unordered_map>

namespace qkv {

namespace {

constexpr int kBK = 64;                           // K per stage: one 128-byte swizzle atom of bf16
constexpr int kBM = 128;                          // weight rows per tile (MMA M)
constexpr uint32_t kABytes = kBM * kBK * 2;       // 16 KB
constexpr int kGemmThreads = 192;

template <int BN> struct TcTraits {
    static constexpr uint32_t kBBytes = BN * kBK * 2;
    static constexpr int NS = BN <= 32 ? 8 : BN <= 64 ? 8 : BN <= 128 ? 6 : 4;
    static constexpr uint32_t kStage = kABytes + kBBytes;
    static constexpr int kCols = BN < 32 ? 32 : BN;  // TMEM columns (power of two >= 32)
    static constexpr size_t kSmem = 1024 /*align slack*/ + static_cast<size_t>(NS) * kStage + 256;
};

struct TcParams {
    int M, N, K;
    int ktiles_per_split;
    float *C;
    int accumulate;   // 0: store (single split) / red.add into a zeroed C; 1: red.add into C
    DevError *err;
};

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

// Instruction descriptor: bf16 x bf16 -> f32, both K-major, M = 128, N = BN.
template <int BN> __device__ __forceinline__ uint32_t idesc_bf16() {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
           (static_cast<uint32_t>(kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, int accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accum)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ bool bounded_wait(uint64_t *bar, uint32_t parity) {
    return mbar_wait(bar, parity, kWaitLimitCycles);
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, TcParams p) {
    using T = TcTraits<BN>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled tiles.
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *tiles = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(tiles + static_cast<size_t>(T::NS) * T::kStage);
    uint64_t *empty = full + T::NS;
    uint64_t *acc_full = empty + T::NS;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
    volatile int *failed = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kBM;
    const int m0 = blockIdx.y * BN;
    const int ktiles = p.K / kBK;
    const int kt0 = blockIdx.z * p.ktiles_per_split;
    const int kt1 = min(ktiles, kt0 + p.ktiles_per_split);
    const int nk = kt1 > kt0 ? kt1 - kt0 : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < T::NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        *failed = 0;
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

    if (warp == 0) {
        if (lane == 0 && nk > 0) {
            const uint64_t pol_w = l2_evict_first_policy();
            const uint64_t pol_x = l2_evict_last_policy();
            int issued = 0;
            for (int i = 0; i < nk; ++i) {
                const int s = i % T::NS;
                const uint32_t ph = static_cast<uint32_t>(i / T::NS) & 1u;
                if (*failed || !bounded_wait(&empty[s], ph ^ 1u)) {
                    report_error(p.err, kErrWaitTimeout, kWhereGemm, blockIdx.x, i);
                    *failed = 1;
                    break;
                }
                uint8_t *a = tiles + static_cast<size_t>(s) * T::kStage;
                uint8_t *b = a + kABytes;
                mbar_arrive_expect_tx(&full[s], T::kStage);
                const int kx = (kt0 + i) * kBK;
                tma_load_2d(a, &tmW, kx, n0, &full[s], pol_w);
                tma_load_2d(b, &tmX, kx, m0, &full[s], pol_x);
                ++issued;
            }
            // Drain: every tile this thread asked for has landed before the CTA can exit.
            for (int i = issued > T::NS ? issued - T::NS : 0; i < issued; ++i) {
                if (!bounded_wait(&full[i % T::NS], static_cast<uint32_t>(i / T::NS) & 1u)) {
                    report_error(p.err, kErrWaitTimeout, kWhereGemm, blockIdx.x, -(1 << 21));
                    break;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16<BN>();
            int issued = 0;
            for (int i = 0; i < nk; ++i) {
                const int s = i % T::NS;
                const uint32_t ph = static_cast<uint32_t>(i / T::NS) & 1u;
                if (*failed || !bounded_wait(&full[s], ph)) {
                    report_error(p.err, kErrWaitTimeout, kWhereGemm, blockIdx.x, -1 - i);
                    *failed = 1;
                    break;
                }
                tc_fence_after();
                const uint8_t *a = tiles + static_cast<size_t>(s) * T::kStage;
                const uint8_t *b = a + kABytes;
                const uint64_t da = smem_desc_sw128(a), db = smem_desc_sw128(b);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    // advance 16 bf16 = 32 bytes inside the swizzle atom (descriptor units of 16 B)
                    mma_bf16(tmem, da + 2ull * kk, db + 2ull * kk, idesc, (i > 0 || kk > 0) ? 1 : 0);
                }
                mma_commit(&empty[s]);
                ++issued;
            }
            // acc_full completes only when every MMA this thread issued has finished,
            // also on the failure path (TMEM is freed after the epilogue saw it).
            if (issued > 0) mma_commit(acc_full);
            else mbar_arrive(acc_full);
        }
        __syncwarp();
    } else {
        // epilogue: warps 2..5, TMEM lanes 32*(warp%4) .. +31 = weight rows of this tile
        const int q = warp & 3;
        const int row = 32 * q + lane;
        const int n = n0 + row;
        const bool have = bounded_wait(acc_full, 0);
        if (!have) report_error(p.err, kErrWaitTimeout, kWhereGemm, blockIdx.x, 1 << 20);
        tc_fence_after();
        // Warp-uniform: tcgen05.ld is .sync.aligned, every lane of the warp must issue it.
        const bool valid_acc = __all_sync(0xffffffffu, have && nk > 0 && !*failed);
        const bool atomic = p.accumulate || gridDim.z > 1;
#pragma unroll 1
        for (int c = 0; c < BN; c += 8) {
            float v[8];
            if (valid_acc) {
                tmem_ld8(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(c), v);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = 0.0f;
            }
            if (n < p.N) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int m = m0 + c + j;
                    if (m < p.M) {
                        float *dst = p.C + static_cast<size_t>(m) * p.N + n;
                        if (atomic) {
                            if (valid_acc) atomicAdd(dst, v[j]);
                        } else {
                            *dst = v[j];
                        }
                    }
                }
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

// bf16 matrix [rows][K] (row-major), box = box_rows x 64 with the 128-byte swizzle.
bool make_map(CUtensorMap *m, const void *ptr, int rows, int K, int box_rows) {
    EncodeTiled enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct MapKey {
    const void *ptr;
    int rows, K, box;
    bool operator==(const MapKey &o) const { return ptr == o.ptr && rows == o.rows && K == o.K && box == o.box; }
};
struct MapKeyHash {
    size_t operator()(const MapKey &k) const {
        return std::hash<const void *>()(k.ptr) ^ (static_cast<size_t>(k.rows) * 1000003u) ^
               (static_cast<size_t>(k.K) << 20) ^ static_cast<size_t>(k.box);
    }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

bool cached_map(CUtensorMap *out, const void *ptr, int rows, int K, int box) {
    std::lock_guard<std::mutex> lock(g_map_mu);
    const MapKey key{ptr, rows, K, box};
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
        *out = it->second;
        return true;
    }
    if (g_maps.size() > 4096) g_maps.clear();
    CUtensorMap m;
    if (!make_map(&m, ptr, rows, K, box)) return false;
    g_maps.emplace(key, m);
    *out = m;
    return true;
}

template <int BN> cudaError_t prepare_bn() {
    return cudaFuncSetAttribute(gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(TcTraits<BN>::kSmem));
}

template <int BN>
cudaError_t launch_bn(const void *X, const void *W, float *C, int M, int N, int K, int accumulate, int num_sms,
                      DevError *err, cudaStream_t st) {
    CUtensorMap tw, tx;
    if (!cached_map(&tw, W, N, K, kBM) || !cached_map(&tx, X, M, K, BN)) return cudaErrorInvalidValue;
    const int tiles_n = (N + kBM - 1) / kBM, tiles_m = (M + BN - 1) / BN;
    const int ktiles = K / kBK;
    int splits = 1;
    const int tiles = tiles_n * tiles_m;
    if (tiles < num_sms) {
        splits = (2 * num_sms + tiles - 1) / tiles;
        const int max_splits = ktiles / 2 > 0 ? ktiles / 2 : 1;
        if (splits > max_splits) splits = max_splits;
    }
    const int kps = (ktiles + splits - 1) / splits;
    splits = (ktiles + kps - 1) / kps;
    if (splits > 1 && !accumulate) {
        cudaError_t e = cudaMemsetAsync(C, 0, static_cast<size_t>(M) * N * sizeof(float), st);
        if (e != cudaSuccess) return e;
    }
    TcParams p{M, N, K, kps, C, accumulate, err};
    dim3 grid(tiles_n, tiles_m, splits);
    gemm_tc_kernel<BN><<<grid, kGemmThreads, TcTraits<BN>::kSmem, st>>>(tw, tx, p);
    return cudaGetLastError();
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

cudaError_t launch_gemm_tc(const void *X, const void *W, float *C, int M, int N, int K, int accumulate, int num_sms,
                           DevError *err, cudaStream_t st) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (K % kBK != 0) return cudaErrorInvalidValue;
    if (M <= 32) return launch_bn<32>(X, W, C, M, N, K, accumulate, num_sms, err, st);
    if (M <= 64) return launch_bn<64>(X, W, C, M, N, K, accumulate, num_sms, err, st);
    if (M <= 128) return launch_bn<128>(X, W, C, M, N, K, accumulate, num_sms, err, st);
    return launch_bn<256>(X, W, C, M, N, K, accumulate, num_sms, err, st);
}

}  // namespace qkv
