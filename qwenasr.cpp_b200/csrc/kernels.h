// Kernel parameter blocks and host launch wrappers of the sm_100a kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <utility>

#include "kcommon.cuh"

namespace qkv {

// Programmatic dependent launch of the step kernels (on unless the
// environment sets QWENASR_B200_PDL=0, read once per process).
inline bool pdl_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("QWENASR_B200_PDL");
        return !(v && std::strcmp(v, "0") == 0);
    }();
    return on;
}

// Launch `kernel` allowing it to start while the stream's previous kernel
// finishes (the kernel must pdl_wait before touching that kernel's memory).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// kKvFP8: K and V in e4m3.  kKvE4I8: K in e4m3, V in int8 (excess-128 bytes);
// both one byte per element with an f32 scale per (page, K|V, kv head).
enum KvDtype { kKvF32 = 0, kKvBF16 = 1, kKvFP8 = 2, kKvE4I8 = 3 };
inline bool kv_is_8bit(int kv_dtype) { return kv_dtype == kKvFP8 || kv_dtype == kKvE4I8; }
inline size_t kv_elem_bytes(int kv_dtype) { return kv_dtype == kKvF32 ? 4 : (kv_dtype == kKvBF16 ? 2 : 1); }
enum ActDtype { kActF32 = 0, kActBF16 = 1 };

constexpr int kAttnMaxRows = 1024;   // rows (streams) per decode-attention launch

// Pool layout of one layer: [n_pages][2 (K,V)][kHkv][kPageTokens][kHeadDim]
// elements of the cache dtype; 8-bit scales: [n_pages][2][kHkv][kPageTokens]
// f32, one per stored (token, head) vector: value = code x scale.
struct AppendParams {
    int n;                     // rows
    const int *slots;          // [n] stream ids (page-table rows)
    const int *positions;      // [n] token position of each row
    const float *qkv;          // [n][kQkvDim] raw projections
    float *q_out;              // [n][kQDim] f32, or null
    void *q16_out;             // [n][kQDim] 16-bit q x q16_scale (K3's Q operand), or null
    float q16_scale;
    int q16_f16;               // 1: f16 (e4m3 cache), 0: bf16
    const float *q_norm_w;     // [kHeadDim]
    const float *k_norm_w;     // [kHeadDim]
    const float2 *rope;        // [rope_len][kHeadDim/2] (cos, sin)
    int rope_len;
    void *pool;                // this layer's pool
    float *scales;             // this layer's FP8 scales (or null)
    const int *page_table;     // [max_streams][maxp]
    int maxp;
    int max_streams;
    int n_pages;
    float eps;
    DevError *err;
    int v_int8;                // 8-bit cache: 1 = V stored as int8 (kKvE4I8), 0 = e4m3
    int qkv_slices;            // qkv holds this many partial-sum slices (>= 1), summed in order
    size_t qkv_slice_stride;   // floats between slices
};

struct AttendParams {
    int n;                     // rows (<= kAttnMaxRows)
    const int *slots;          // [n]
    const int *lens;           // [n] tokens to attend over (including the new one)
    const float *q;            // [n][kQDim] post-RoPE queries
    void *out;                 // [n][kQDim] f32 or bf16
    const void *pool;          // this layer's pool
    const float *scales;       // this layer's FP8 scales (or null)
    const int *page_table;
    int maxp;
    int max_streams;
    int n_pages;
    float *part_o;             // [n + grid][kHq][kHeadDim] scratch
    float *part_ml;            // [n + grid][kHq][2] scratch
    int *counters;             // [n][kHkv], zero between launches
    float scale_log2;          // log2(e) / sqrt(head_dim)
    DevError *err;
    // 1: the kernel(s) just before this launch on the stream wrote only each
    // row's LAST page (one new token per row: K1, or the previous layer's K2
    // with the append-ahead), and the row arrays and page table came from
    // copies that finished before them, so K2 may set up and stream the other
    // pages before its grid dependency wait.  0: everything waits (any caller).
    int early;
    // Append-ahead (KV steps, where every layer's projections are on the
    // device before the step starts): with next.n > 0, K2 of layer l also
    // does K1's work for layer l + 1 on its three append warps (rows dealt
    // evenly over the CTAs, after the grid dependency wait), so that layer's
    // pages and q are ready when its K2 starts and no append sits between
    // two attention launches.  next.q_out must not be this launch's q.
    AppendParams next;
};

struct PrefillAttnParams {
    int n;                     // query rows
    const int *slots;          // [n]
    const int *positions;      // [n] query position; keys are [0, position]
    const float *q;            // [n][kQDim] (CUDA-core kernel)
    const void *q16;           // [n][kQDim] q x scale_log2 in bf16 (f16 for e4m3), for K3
    void *out;                 // [n][kQDim] f32 or bf16
    const void *pool;
    const float *scales;
    const int *page_table;
    int maxp;
    int max_streams;
    int n_pages;
    float scale_log2;
    DevError *err;
};

cudaError_t launch_kv_append(const AppendParams &p, int kv_dtype, cudaStream_t st);
cudaError_t prepare_decode_attn();
size_t attn_smem_bytes(int kv_dtype);
cudaError_t launch_decode_attn(const AttendParams &p, int kv_dtype, bool out_bf16, int grid, cudaStream_t st);
// Read probe of K2's page stream: pages[0..n) (ids into this layer's pool of
// n_pool_pages pages of page_bytes <= 64 KB) bulk-copied into shared memory and
// discarded, split over `grid` persistent CTAs like K2's page list.
cudaError_t launch_page_read_probe(const void *pool_layer, uint32_t page_bytes, const int *pages, int n,
                                   int n_pool_pages, int grid, DevError *err, cudaStream_t st);
// Test of the bounded waits: one CTA whose waits (K2's stage and hand-over
// waits, the plain mbarrier wait) run out after limit_cycles and report it.
cudaError_t launch_wait_probe(DevError *err, long long limit_cycles, cudaStream_t st);
cudaError_t launch_prefill_attn(const PrefillAttnParams &p, int kv_dtype, bool out_bf16, cudaStream_t st);
// K3 (bf16 or e4m3 cache): items = (first row, query count <= 64, kv head, 0), one CTA each.
cudaError_t prepare_prefill_tc();
bool prefill_tc_supported(int kv_dtype);
cudaError_t launch_prefill_attn_tc(const PrefillAttnParams &p, int kv_dtype, const int4 *items, int n_items,
                                   bool out_bf16, cudaStream_t st);
// q (f32, [n][kQDim]) x scale rounded to bf16 (f16 if `f16`): K3's Q operand for callers that hold f32 q.
cudaError_t launch_q_to16(const float *q, int n, float scale, bool f16, void *out, cudaStream_t st);
cudaError_t launch_page_gather(const void *pool, int kv_dtype, const int *pages, int n_pages_row, int len,
                               int n_pages, void *k_out, void *v_out, DevError *err, cudaStream_t st);
cudaError_t launch_page_copy(void *pool_layer, size_t page_bytes, const int *src, const int *dst, int n,
                             cudaStream_t st);
cudaError_t launch_page_fill(void *pool_layer, float *scales_layer, int kv_dtype, const int *pages, int n,
                             uint64_t seed, cudaStream_t st);

// ---- dense kernels ----
// out[r] = rmsnorm(x[rows? rows[r] : r]) * w   (double mean square, as text-decoder.cpp:542-557)
// Split-K partial sums of the projection that produced the residual rows
// (the GEMM's slice mode), folded in by the kernel that reads those rows
// next: x[r] += slices[s][r] for s = 0, 1, ... n - 1 in that order (slices
// indexed like x, `stride` floats apart), the sum written back into x.
// n == 0: nothing to fold.
struct ResidualFold {
    const float *slices = nullptr;
    int n = 0;
    size_t stride = 0;
};

cudaError_t launch_rmsnorm(float *x, const int *rows, int n, int hidden, const float *w, float eps,
                           void *out, int out_dtype, cudaStream_t st, ResidualFold fold = {});
// x[r] (+)= fold, rows 0..n-1 of width hidden.
cudaError_t launch_residual_fold(float *x, int n, int hidden, ResidualFold fold, cudaStream_t st);
// x[r] = embd[ids[r]] as f32
// Audio projector pieces: LayerNorm (weight, bias) of f32 rows into `out_dtype`;
// out = act(c + bias) (act = erf GELU or identity) into `out_dtype`.
cudaError_t launch_layernorm(const float *x, int n, int width, const float *w, const float *b, float eps, void *out,
                             int out_dtype, cudaStream_t st);
cudaError_t launch_bias_act(const float *c, const float *bias, int n, int width, bool gelu, void *out, int out_dtype,
                            cudaStream_t st);
// Prompt rows from ids: embedding row of ids[t], or audio row rows[src[t]] where src[t] >= 0.
cudaError_t launch_decoder_input(const int *ids, const int *src, int n, const void *embd, int w_dtype, int hidden,
                                 const float *const *rows, float *x, cudaStream_t st);
cudaError_t launch_embed(const int *ids, int n, const void *embd, int w_dtype, int hidden, int vocab, float *x,
                         DevError *err, cudaStream_t st);
// C[m][n] (+)= sum_k X[m][k] * W[n][k];  X: act dtype, W: weight dtype, C f32.
// epilogue 0: store, 1: accumulate into C (residual add).
cudaError_t launch_gemm(const void *X, int x_dtype, const void *W, int w_dtype, float *C, int M, int N, int K,
                        int epilogue, cudaStream_t st);
// tcgen05 path (bf16 X and W, K % 64 == 0): C (+)= X . W^T, split-K with f32
// red.add when the tile grid is smaller than the SM count.
cudaError_t prepare_gemm_tc();
bool gemm_tc_supported(int M, int N, int K);
// act[M][N2/2] (bf16) = silu(gate) * up of X . W^T, W = gate/up rows
// interleaved one by one (row 2f gate f, row 2f + 1 up f; N2 even); one K split.
// With a workspace (sk_ws of sk_ws_floats f32, sk_flags of 4 x sk_flag_tiles
// ints, zero before first use and left zero) a launch whose tiles would leave
// SMs idle runs stream-K over all of them (see TcParams).  Calls sharing a
// workspace must not overlap.
cudaError_t launch_gemm_tc_swiglu(const void *X, const void *W, void *act, int M, int N2, int K, int num_sms,
                                  DevError *err, cudaStream_t st, float *sk_ws = nullptr, int *sk_flags = nullptr,
                                  size_t sk_ws_floats = 0, int sk_flag_tiles = 0);
bool gemm_tc_swiglu_pays(int M, int N2, int K, int num_sms);
// Kernels one launch_gemm_tc call launches: 2 when a K split first zeroes C.
int gemm_tc_kernels(int M, int N, int K, int accumulate, int num_sms);
// FP8 projections (tcgen05 kind::f8f6f4, e4m3 x e4m3 -> f32, K % 128 == 0):
// C (+)= (X x x_scale[m]) . (W x w_scale[n])^T with one scale per token row
// of X and per weight row of W; same tiling, split and epilogues as bf16.
// Slice mode: C = X . W^T as *slices partial products (one per K split, at
// most max_slices) in C[s][M][N]; the reader sums them in slice order.  No
// zeroing kernel, no atomics; C must hold max_slices x M x N floats.
cudaError_t launch_gemm_tc_slices(const void *X, const void *W, float *C, int M, int N, int K, int max_slices,
                                  int num_sms, DevError *err, cudaStream_t st, int *slices);
cudaError_t launch_gemm_tc_fp8_slices(const void *X, const float *x_scale, const void *W, const float *w_scale,
                                      float *C, int M, int N, int K, int max_slices, int num_sms, DevError *err,
                                      cudaStream_t st, int *slices);
bool gemm_tc_fp8_supported(int M, int N, int K);
int gemm_tc_fp8_kernels(int M, int N, int K, int accumulate, int num_sms);
cudaError_t launch_gemm_tc_fp8(const void *X, const float *x_scale, const void *W, const float *w_scale, float *C,
                               int M, int N, int K, int accumulate, int num_sms, DevError *err, cudaStream_t st);
// Rows -> e4m3 codes + one f32 scale per row (amax / 448): mode 0 bf16 rows,
// 1 RMSNorm(f32 rows) x w, 2 SwiGLU of f32 gate/up rows [n][2K] interleaved one by one.
int rows_q8_max_k();   // widest row the quantiser takes (6144)
cudaError_t launch_rows_q8(int mode, const void *in, int n, int K, const float *w, float eps, void *out, float *scales,
                           cudaStream_t st, ResidualFold fold = {});
cudaError_t launch_gemm_tc(const void *X, const void *W, float *C, int M, int N, int K, int accumulate, int num_sms,
                           DevError *err, cudaStream_t st);
// Shared-memory opt-in of the dense kernels for rows up to max_k wide.
cudaError_t prepare_dense(int max_k);
// out[m][j] = silu(gu[m][j]) * gu[m][F + j]
cudaError_t launch_swiglu(const float *gu, int M, int F, void *out, int out_dtype, cudaStream_t st);
// GGUF tensor data (ggml type 0 f32, 1 f16, 30 bf16 passed as 2) -> weight dtype.
cudaError_t launch_convert(const void *src, int src_ggml_type, void *dst, int dst_dtype, size_t n, cudaStream_t st);
// ids[m] = first index of the maximum of logits[m][0..V)
// Row argmax (the first maximum; NaN never wins) with each row split over up
// to max_slices CTAs (grid about two waves); part_v / part_i [M][max_slices]
// scratch, counters [M] zero between launches (the kernel resets them).
cudaError_t launch_argmax_split(const float *logits, int M, int V, int *ids, float *part_v, int *part_i,
                                int *counters, int max_slices, int num_sms, cudaStream_t st);
// bf16 LM head: the largest row norm of W (once, at load), and the exact
// re-scoring of every token whose approximate logit could be the f32 maximum
// (keys/counters: [M] zeroed once; they reset themselves).
cudaError_t launch_row_norm_max(const void *W, int rows, int H, float *out, cudaStream_t st);
cudaError_t launch_argmax_refine(const float *logits, int M, int V, const float *x, const int *rows, int H,
                                 const float *norm_w, float eps, const void *W, const float *wmax,
                                 unsigned long long *keys, int *counters, int *ids, int num_sms, cudaStream_t st);

}  // namespace qkv
