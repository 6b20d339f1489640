// The handle behind the C ABI: one CUDA device, its weights, its paged KV pool
// and stream table, and the per-step scratch.  Replaces the reference's
// QwenAsrTextDecoderBackend (text-decoder.cpp:165-189): weights are uploaded
// once at create (:1476-1592), the cache is a page pool instead of one
// contiguous max_seq_len tensor per layer (:1420-1474), and every forward is a
// fixed sequence of kernel launches instead of a GGML graph rebuilt per call
// (:1641-1755).
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <string>
#include <tuple>
#include <vector>

#include "kernels.h"
#include "pager.h"
#include "qkv.h"

struct qkv_handle {
    struct Layer {
        float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
        void *w_qkv = nullptr;   // [(Hq+2Hkv)D][H]  q rows, then k rows, then v rows
        void *w_o = nullptr;     // [H][Hq D]
        void *w_gu = nullptr;    // [2F][H]  gate rows, then up rows
        void *w_down = nullptr;  // [H][F]
        // FP8 projections: one f32 scale per weight row (the codes are in w_*)
        float *s_qkv = nullptr, *s_o = nullptr, *s_gu = nullptr, *s_down = nullptr;
    };

    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    qkv_model_config cfg{};
    qkv_runtime_config rt{};
    bool has_weights = false;
    int w_dtype = 0;     // kActF32 / kActBF16 (weights and GEMM inputs)
    int act_dtype = 0;   // activations feeding GEMMs
    size_t w_elem = 4;

    std::vector<Layer> layers;
    void *embd = nullptr;      // [V][H]
    void *w_out = nullptr;     // [V][H]
    float *out_norm = nullptr; // [H]
    // Audio projector (optional in the GGUF): LayerNorm [Ha] weight/bias, proj0
    // [Ha][Ha] + bias, proj1 [H][Ha] + bias (weights in the weight dtype).
    int audio_hidden = 0;
    float *ap_norm_w = nullptr, *ap_norm_b = nullptr, *ap_b0 = nullptr, *ap_b1 = nullptr;
    void *ap_w0 = nullptr, *ap_w1 = nullptr;

    // KV pool
    void *pool = nullptr;
    size_t pool_layer_bytes = 0;
    size_t page_bytes = 0;      // one page of one layer
    float *scales = nullptr;    // FP8: [L][n_pages][2][Hkv]
    size_t scales_layer_elems = 0;
    int n_pages = 0;
    int maxp = 0;               // pages per stream
    int *d_page_table = nullptr;
    int *h_page_table = nullptr;    // pinned mirror [max_streams][maxp]
    float2 *d_rope = nullptr;
    int rope_len = 0;
    qkv::Pager *pager = nullptr;

    // scratch (rows = max(max_batch_tokens, max_streams))
    int max_rows = 0;
    float *x = nullptr, *qkv = nullptr, *q = nullptr, *gu = nullptr, *logits = nullptr;
    float *q_alt = nullptr;   // [max_streams][kQDim]: the second q buffer of the KV step's append-ahead
    float *host_stage = nullptr;    // device staging of qkv_kv_step_host
    size_t host_stage_bytes = 0;
    void *xn = nullptr, *attn = nullptr, *act = nullptr;
    int *d_rowbuf = nullptr;    // [4][max_rows]: slots, positions, lens, ids
    int *h_rowbuf = nullptr;    // pinned staging, kRowRing slots of [4][max_rows]
    static constexpr int kRowRing = 4;
    cudaEvent_t row_ev[kRowRing] = {};   // recorded after the copy out of each slot
    cudaEvent_t items_ev = nullptr;      // recorded after the copy out of h_items
    int row_slot = 0;
    // Prompt embeddings go to the device through kEmbRing pinned chunks of
    // kEmbChunkBytes: host threads fill a chunk, one asynchronous copy moves
    // it, and a chunk is refilled only after its copy has run (its event).
    static constexpr int kEmbRing = 2;
    static constexpr size_t kEmbChunkBytes = size_t(16) << 20;
    float *h_emb[kEmbRing] = {};
    cudaEvent_t emb_ev[kEmbRing] = {};
    int emb_slot = 0;
    // Decoder input from ids: pinned / device staging of [ids | row source]
    // ([2][max_rows] int32) and of the audio-row pointer table ([max_rows]),
    // rewritten only after the copies that last read them have run (dec_ev).
    int *h_dec = nullptr, *d_dec = nullptr;
    const float **h_rowptr = nullptr, **d_rowptr = nullptr;
    cudaEvent_t dec_ev = nullptr;
    // qkv_kv_step_host's per-layer pipeline: inputs go up on copy_in, outputs
    // come back on copy_out, one event per layer each way (created on first use).
    cudaStream_t copy_in = nullptr, copy_out = nullptr;
    std::vector<cudaEvent_t> ev_in, ev_done;
    cudaEvent_t ev_tail = nullptr;
    // split argmax scratch: partials [max_streams][kArgmaxSlices], per-row counters (zero between launches)
    static constexpr int kArgmaxSlices = 16;
    float *am_v = nullptr;
    int *am_i = nullptr, *am_cnt = nullptr;
    // exact re-scoring of the bf16 head's argmax: per-row keys and counters
    // (zero between launches) and the largest row norm of the head weights
    unsigned long long *am_keys = nullptr;
    int *am_rcnt = nullptr;
    float *d_wout_norm = nullptr;
    bool exact_argmax = true;   // QWENASR_B200_EXACT_ARGMAX=0 turns the re-scoring off
    // weight_dtype QKV_FP8_E4M3: the four projections hold e4m3 codes with a
    // scale per weight row and take e4m3 token rows with a scale per row (xq,
    // xq_s); embeddings, the LM head and the audio projector stay bf16.
    bool proj_fp8 = false;
    // qkv projection of a decode-sized batch in slice mode: one partial sum per
    // K split in qkv_sl[s][rows][kQkvDim], summed in order by K1 (no zeroing
    // kernel, no atomics, deterministic).
    static constexpr int kQkvMaxSlices = 8;
    float *qkv_sl = nullptr;
    int qkv_nsl = 1;
    size_t qkv_sl_stride = 0;
    // o and down projections of a decode-sized batch in slice mode: the split
    // partial sums go to res_sl[s][rows][H] and the next RMSNorm (or the
    // head's) adds them to the residual x in slice order; res_pending is the
    // last layer's down projection, still to be folded by the head.
    // Off by default (QWENASR_B200_RESIDUAL_SLICES=1 turns it on): it keeps
    // atomics out of the residual, but the folds cost the RMSNorms more than
    // the red.add they replace (measured 2-4 % per decode step).
    static constexpr int kResMaxSlices = 8;
    float *res_sl = nullptr;
    bool res_slices = false;
    qkv::ResidualFold res_pending;
    // Stream-K workspace of the fused gate/up GEMM at decode batches (partial
    // tiles and per-tile counters, the counters zero between launches).
    float *sk_ws = nullptr;
    int *sk_flags = nullptr;
    size_t sk_ws_floats = 0;
    int sk_flag_tiles = 0;
    // QWENASR_B200_STREAM_K=1 spreads a decode batch's fused gate/up GEMM over
    // all SMs (stream-K); off by default: measured 3-5 % slower per decode step.
    bool stream_k = false;
    uint8_t *xq = nullptr;      // [rows][max(H, Hq D, F)] e4m3 token operand
    float *xq_s = nullptr;      // [rows]
    int *d_out_ids = nullptr;   // [max_rows]
    int *h_out_ids = nullptr;   // pinned
    int4 *d_items = nullptr;    // prefill attention work items
    int4 *h_items = nullptr;    // pinned
    int max_items = 0;
    float *part_o = nullptr, *part_ml = nullptr;
    int *counters = nullptr;
    qkv::DevError *d_err = nullptr;
    qkv::DevError *h_err = nullptr;
    std::vector<int32_t> last_id;   // per slot: last greedy id

    std::string last_error;
    int64_t launches = 0;

    // Captured device work, replayed each call: decode step per batch size,
    // microbench KV step per (batch size, qkv buffer, out buffer).
    struct Graph {
        cudaGraphExec_t exec = nullptr;
        int64_t kernels = 0;
    };
    std::map<int, Graph> decode_graphs;
    std::map<std::tuple<int, const void *, const void *>, Graph> kv_graphs;
    // Host-buffer KV steps with pinned buffers: (rows, qkv_host, out_host, staging) -> graph.
    std::map<std::tuple<int, const void *, const void *, const void *>, Graph> kvh_graphs;
    bool use_graphs = true;
    // Prefill attention on the tensor cores (K3) for bf16/e4m3 caches; the
    // environment variable QWENASR_B200_PREFILL_ATTN=cuda_core selects the
    // CUDA-core kernel instead (a cross-check of the two device paths).
    bool prefill_tc = true;
    // SwiGLU in the gate/up GEMM's epilogue where each CTA gets >= 2 work
    // units (QWENASR_B200_FUSED_SWIGLU=0: the separate SwiGLU kernel).
    bool fused_swiglu = true;
    // KV steps: K2 of layer l also appends layer l + 1 (AttendParams::next),
    // so the step is K1 of layer 0 and one launch per layer
    // (QWENASR_B200_APPEND_AHEAD=0: K1 then K2 for every layer).
    bool append_ahead = true;
    int last_decode_n = -1;   // a graph is captured only for a batch size seen twice in a row
};

namespace qkv {
// Status helpers shared by the C ABI implementation files.
int fail(qkv_handle *h, int code, const std::string &msg);
int cuda_fail(qkv_handle *h, cudaError_t e, const char *what);
}  // namespace qkv
