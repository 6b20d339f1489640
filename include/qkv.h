/*
 * qkv.h -- C ABI of the B200 (sm_100a) Qwen3-ASR text-decoder KV-cache path.
 *
 * This is the drop-in boundary for the reference's decoder operator surface
 * (qwenasr.cpp src/text-decoder.h).  All entry points are extern "C", take
 * plain pointers and sizes, and return an int status (QKV_OK == 0).  A handle
 * owns one CUDA device: its weights, its paged KV pool and its stream table.
 * It is driven by one host thread at a time.  Multi-GPU = one handle per GPU.
 *
 * Every entry point whose arguments are host buffers runs on the handle's own
 * CUDA stream and synchronises it before it returns.  Entry points taking
 * device pointers run on the CUDA stream passed in (NULL = the legacy default
 * stream) and do not synchronise.
 *
 * Errors: a non-zero status; the message is kept per handle and read with
 * qkv_last_error().  Kernels never trap: device-side failures (a bounded wait
 * that ran out, an out-of-range page index) set a device error word that the
 * next synchronising call turns into QKV_ERR_DEVICE.
 */
#ifndef QKV_H
#define QKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QKV_ABI_VERSION 1

typedef struct qkv_handle qkv_handle;
typedef struct qkv_tokenizer qkv_tokenizer;
typedef struct qkv_pager qkv_pager;

enum qkv_status {
    QKV_OK = 0,
    QKV_ERR_INVALID_ARG = 1,   /* bad argument or configuration */
    QKV_ERR_OUT_OF_PAGES = 2,  /* the KV pool has no free page */
    QKV_ERR_CAPACITY = 3,      /* stream / context / batch limit exceeded */
    QKV_ERR_CUDA = 4,          /* a CUDA runtime call failed */
    QKV_ERR_DEVICE = 5,        /* a kernel reported an error (bounds, bounded wait) */
    QKV_ERR_IO = 6,            /* file could not be opened / mapped */
    QKV_ERR_FORMAT = 7,        /* GGUF parse error, missing tensor, shape or type mismatch */
    QKV_ERR_STATE = 8,         /* call not valid in the current state */
    QKV_ERR_NO_DEVICE = 9,     /* no CUDA device / wrong architecture */
    QKV_ERR_HOST_MEMORY = 10   /* a host table or string did not fit in host memory */
};

enum qkv_dtype {
    QKV_F32 = 0,
    QKV_BF16 = 1,
    QKV_FP8_E4M3 = 2,          /* KV cache only: e4m3 values; fp32 scale per stored (token, kv head)
                                  vector of K and of V: [n_pages][2][8][16], value = code x scale */
    QKV_E4M3K_I8V = 3          /* KV cache only: K in e4m3, V in int8 stored as excess-128 bytes
                                  (byte u holds (u - 128) x scale); scales as for QKV_FP8_E4M3 */
};

/* Decoder hyper-parameters (GGUF keys qwen3-asr.text.*).
 * Mirrors the int/float parameters of qwenasr_text_decoder_backend_init
 * (text-decoder.h:85-99). */
typedef struct qkv_model_config {
    int32_t n_layers;
    int32_t hidden;
    int32_t n_heads;
    int32_t n_kv_heads;
    int32_t head_dim;        /* must be 128 */
    int32_t intermediate;
    int32_t vocab;
    float rope_theta;
    float rms_norm_eps;
} qkv_model_config;

/* Runtime / memory plan of a handle.  Replaces the reference's single
 * max_seq_len (text-decoder.h:101-116) with a paged pool. */
typedef struct qkv_runtime_config {
    int32_t device;            /* CUDA device ordinal */
    int32_t weight_dtype;      /* QKV_F32, QKV_BF16 (f32 GGUF values are rounded RNE) or
                                  QKV_FP8_E4M3: the four projections of every layer in e4m3
                                  with one f32 scale per weight row, their inputs quantised to
                                  e4m3 per token row (embeddings, LM head: bf16) */
    int32_t kv_dtype;          /* QKV_F32, QKV_BF16, QKV_FP8_E4M3 or QKV_E4M3K_I8V */
    int32_t page_tokens;       /* tokens per page; must be 16 */
    int32_t max_streams;       /* stream slots */
    int32_t max_context;       /* tokens per stream (prompt + generated) */
    int64_t max_pages;         /* pages in the pool; 0 = max_streams * ceil(max_context/page_tokens) */
    int32_t max_batch_tokens;  /* prompt tokens one qkv_prefill call may carry; 0 = max_context */
    uint32_t page_order_seed;  /* 0: pages handed out in pool order; else a seeded permutation */
} qkv_runtime_config;

/* Fill *cfg from the qwen3-asr.text.* keys of a GGUF file
 * (the reference reads them in native-model.cpp:187-218). */
int qkv_read_gguf_config(const char *gguf_path, qkv_model_config *cfg, char *err, size_t err_len);

/* Load the decoder weights of a GGUF file onto rt->device and allocate the KV
 * pool.  Replaces qwenasr_text_decoder_backend_init / _init_cached
 * (text-decoder.h:85-116, text-decoder.cpp:1476-1639).  cfg may be NULL, in
 * which case it is read from the file.  Tensors must be F32, F16 or BF16 with
 * the reference's names and shapes (text-decoder.cpp:191-228, 523-537).  The
 * file is not needed after the call returns.  QKV_ERR_HOST_MEMORY when the
 * host tables a runtime config asks for do not fit in host memory (as for
 * qkv_create_kv_only). */
int qkv_create(const char *gguf_path, const qkv_model_config *cfg, const qkv_runtime_config *rt,
               qkv_handle **out, char *err, size_t err_len);

/* A handle with a KV pool and the per-layer QK-norm weights only (no
 * projection weights): the operator-level entry points below work on it.
 * q_norm_w / k_norm_w are host arrays [n_layers][head_dim]. */
int qkv_create_kv_only(const qkv_model_config *cfg, const qkv_runtime_config *rt,
                       const float *q_norm_w, const float *k_norm_w, qkv_handle **out, char *err,
                       size_t err_len);

/* Replaces qwenasr_text_decoder_backend_free (text-decoder.h:118). NULL-safe. */
void qkv_destroy(qkv_handle *h);

const char *qkv_last_error(const qkv_handle *h);

/* ---- stream table (the reference keeps one stream: cur_len, text-decoder.cpp:186) ---- */
int qkv_stream_open(qkv_handle *h, int32_t *stream_id);
int qkv_stream_close(qkv_handle *h, int32_t stream_id);           /* frees the stream's pages */
int qkv_stream_length(const qkv_handle *h, int32_t stream_id, int32_t *tokens);
int qkv_pool_stats(const qkv_handle *h, int64_t *free_pages, int64_t *total_pages);
/* Move live pages to the low end of the pool (device page copies + page-table
 * rewrite); *moved = pages moved. */
int qkv_compact(qkv_handle *h, int64_t *moved);

/* ---- model-level path (host buffers; synchronising) ---- */

/* Prefill n streams (each must be open and empty) with their prompt rows
 * embeddings[Σ lens][hidden] f32 (audio rows already spliced in, the layout of
 * QwenAsrDecoderInputOutput::values, decoder-input.h:11-17), positions 0..len-1.
 * Writes every layer's K/V into the streams' pages and the greedy id of each
 * stream's last row to out_ids[n].  out_logits (nullable) receives [n][vocab]
 * f32.  Replaces the prefill half of text_decoder_backend_cached_logits
 * (text-decoder.cpp:1641-1755) and qwenasr_text_prefill_backend_forward
 * (:1757-1854). */
int qkv_prefill(qkv_handle *h, int32_t n, const int32_t *stream_ids, const int32_t *lens,
                const float *embeddings, int32_t *out_ids, float *out_logits);

/* qkv_prefill with each stream's prompt rows in a block of its own:
 * embeddings[i] points to lens[i] x hidden f32 host values, so a caller that
 * holds one array per request need not first copy them into one block.  The
 * rows reach the device through the handle's pinned chunks, filled by several
 * host threads (as in qkv_prefill).  The same operation as the prefill half of
 * text_decoder_backend_cached_logits (text-decoder.cpp:1641-1755). */
int qkv_prefill_rows(qkv_handle *h, int32_t n, const int32_t *stream_ids, const int32_t *lens,
                     const float *const *embeddings, int32_t *out_ids, float *out_logits);

/* Audio projector on the device (src/audio-encoder.cpp:848-856, the stage
 * between the audio encoder and the decoder input): rows of the encoder's
 * output, audio_dev [n][Ha] f32 (device), go through LayerNorm (eps 1e-5,
 * weight and bias) -> audio.proj.0 + bias -> erf GELU -> audio.proj.1 + bias
 * into out_dev [n][hidden] f32 (device), on `stream`; the result can go to
 * qkv_prefill_ids / qkv_decoder_input with audio_on_device = 1.  Needs the
 * audio.post_norm / audio.proj tensors in the model file (QKV_ERR_STATE when
 * absent; qkv_audio_projector_width gives Ha, 0 without them).  Uses the
 * handle's prefill scratch: do not overlap it with other calls on the handle. */
int qkv_audio_project(qkv_handle *h, int32_t n, const float *audio_dev, float *out_dev, void *stream);
int qkv_audio_projector_width(const qkv_handle *h, int32_t *width);

/* Decoder input on the device: the embedding lookup and audio-row splice of
 * qwenasr_decoder_input_from_audio (src/decoder-input.cpp:64-98), after the
 * prompt (src/tokenizer.cpp:529-549) has been tokenised by the caller.  For n
 * prompts of lens[i] ids each (ids: sum lens int32, host), row t of the
 * output is the embedding row of ids[t], or, where ids[t] == audio_token_id,
 * the prompt's next audio row: audio[i] points to audio_tokens[i] x hidden
 * f32 values, in host memory, or in device memory when audio_on_device (as
 * an audio encoder on the GPU leaves them).  The same checks and messages as
 * the reference, in its order (QKV_ERR_INVALID_ARG): an id outside the
 * embedding table, more placeholders than audio rows, a count that differs.
 * x_dev: sum lens x hidden f32 (device), written on `stream`.  The embedding
 * rows are the handle's table (bf16-rounded in bf16 weight mode). */
int qkv_decoder_input(qkv_handle *h, int32_t n, const int32_t *lens, const int32_t *ids,
                      const float *const *audio, const int32_t *audio_tokens, int32_t audio_on_device,
                      int32_t audio_token_id, float *x_dev, void *stream);

/* qkv_prefill with the prompt rows built on the device by qkv_decoder_input
 * (arguments as there): only the ids and the audio rows cross to the device,
 * and nothing does when the audio rows are already there. */
int qkv_prefill_ids(qkv_handle *h, int32_t n, const int32_t *stream_ids, const int32_t *lens, const int32_t *ids,
                    const float *const *audio, const int32_t *audio_tokens, int32_t audio_on_device,
                    int32_t audio_token_id, int32_t *out_ids, float *out_logits);

/* One greedy decode step for n streams: embed in_ids (NULL = each stream's
 * last greedy id kept on the device), run all layers appending one token per
 * stream, and write the next greedy ids to out_ids[n] (first maximum, as
 * text-decoder.cpp:2266-2274).  out_logits nullable [n][vocab]. */
int qkv_decode_step(qkv_handle *h, int32_t n, const int32_t *stream_ids, const int32_t *in_ids,
                    int32_t *out_ids, float *out_logits);

/* The reference's cached greedy loop for one stream: prefill, then up to
 * max_new_tokens-1 decode steps, stopping after an id in stop_ids.  Uses (and
 * closes) a temporary stream.  Replaces qwenasr_text_generate_cached_backend
 * (text-decoder.h:156-163, text-decoder.cpp:2209-2311). */
int qkv_generate(qkv_handle *h, const float *embeddings, int32_t tokens, int32_t max_new_tokens,
                 const int32_t *stop_ids, int32_t n_stop, int32_t *out_ids, int32_t *n_out,
                 int32_t *stopped);

/* One decoder block over `tokens` rows at positions 0..tokens-1, no cache
 * kept (a temporary stream is used and closed): x[tokens][hidden] f32 in,
 * out[tokens][hidden] f32.  The single-layer parity probe, replacing
 * qwenasr_text_layer_backend_forward (text-decoder.h:79-83, :1305-1390). */
int qkv_layer_forward(qkv_handle *h, int32_t layer, int32_t tokens, const float *x, float *out);

/* ---- operator level: one layer's K/V append and decode attention ----
 * Device pointers; `stream` is the cudaStream_t to launch on (NULL = the CUDA
 * legacy default stream, as in the CUDA runtime API).  Consecutive calls on a
 * handle must use the same stream (its per-call row staging is stream-ordered).
 * Rows: slots[i] is an open stream id, positions[i] its token position. */

/* K1: qkv[n][Hq*D + 2*Hkv*D] f32 (raw projections) -> QK-RMSNorm + NEOX RoPE;
 * K, V stored into the page of (slot, position); q_out[n][Hq*D] f32.
 * Replaces text-decoder.cpp:375-433 (norm, rope, cpy into the cache view). */
int qkv_kv_append(qkv_handle *h, int32_t layer, int32_t n, const int32_t *slots_dev,
                  const int32_t *positions_dev, const float *qkv_dev, float *q_out_dev, void *stream);

/* K2: decode attention of q[n][Hq*D] f32 over tokens [0, lens[i]) of each
 * row's pages; out[n][Hq*D] f32.  Replaces text-decoder.cpp:435-463. */
int qkv_kv_attend(qkv_handle *h, int32_t layer, int32_t n, const int32_t *slots_dev,
                  const int32_t *lens_dev, const float *q_dev, float *out_dev, void *stream);

/* Operator: C[m][n] (+)= X[m][k] . W[n][k]^T on the tensor cores (tcgen05,
 * bf16 X and W row-major, f32 C; k a multiple of 64).  accumulate = 0 stores,
 * 1 adds into C.  The decoder's projections (text-decoder.cpp:371-373, 465,
 * 469-472, 476-493).  Device pointers, current device, `stream` as above. */
int qkv_gemm_bf16(const void *x, const void *w, float *c, int32_t m, int32_t n, int32_t k, int32_t accumulate,
                  void *stream);

/* Operator: the gate/up projection with SwiGLU in the GEMM's epilogue, on
 * the tensor cores: act[m][n2/2] (bf16) = silu(G) * U, with G and U the rows
 * of X[m][k] . W^T (bf16 in, f32 accumulation) for W[n2][k] (bf16) holding
 * gate and up rows interleaved one by one (row 2f = gate feature f, row 2f + 1
 * = up feature f); n2 even, k a multiple of 64.  silu(g) = g / (1 + exp(-g)),
 * product rounded once to bf16.  Replaces the reference's gate and up
 * mul_mat, ggml_silu and ggml_mul (text-decoder.cpp:476-493).  Optional
 * stream-K workspace (both NULL: none): `workspace` of workspace_floats f32
 * and `flags` of 4 x flag_tiles int32, zero before the first call and left
 * zero by every call; with it, a small batch whose output tiles would leave
 * SMs idle spreads all of their k-tiles evenly over the SMs.  Calls sharing
 * a workspace must not overlap.  Device pointers, current device, `stream`
 * as above. */
int qkv_gemm_swiglu_bf16(const void *x, const void *w, void *act, int32_t m, int32_t n2, int32_t k, float *workspace,
                         int32_t *flags, int64_t workspace_floats, int32_t flag_tiles, void *stream);

/* Operator: the FP8 form of the projections, on the tensor cores (tcgen05
 * kind::f8f6f4, e4m3 x e4m3 products accumulated in f32): C[m][n] (+)=
 * (X[m][k] x x_scale[m]) . (W[n][k] x w_scale[n])^T, X and W e4m3 codes
 * row-major, one f32 scale per row of each; k a multiple of 128.  A
 * B200-side weight format with no counterpart in the reference, whose
 * projections are f32 (text-decoder.cpp:371-373, 465, 469-472).  Device
 * pointers, current device, `stream` as above. */
int qkv_gemm_fp8(const void *x, const float *x_scale, const void *w, const float *w_scale, float *c, int32_t m,
                 int32_t n, int32_t k, int32_t accumulate, void *stream);

/* Rows of bf16 values [rows][k] -> e4m3 codes [rows][k] and one f32 scale per
 * row (amax / 448; 1 for an all-zero row): the quantiser the FP8 weights and
 * token rows go through; k a multiple of 4, at most 6144.  Device pointers,
 * `stream` as above. */
int qkv_quantize_rows_e4m3(const void *x_bf16, int32_t rows, int32_t k, void *codes, float *scales, void *stream);

/* Causal prefill attention over one layer's paged cache (K3 on tcgen05 for
 * bf16/e4m3 caches, the CUDA-core kernel for f32): for each of the n streams
 * the queries are its LAST lens[i] cached positions (the prompt rows just
 * appended), attending to every key at or before their position.  q_dev
 * [sum lens][Hq*D] f32 post-RoPE, rows in stream order; out_dev same shape f32.
 * stream_ids / lens are host arrays.  The prompt half of
 * text-decoder.cpp:322-334 (QK^T, diag mask, softmax, PV), as an operator. */
int qkv_prefill_attend(qkv_handle *h, int32_t layer, int32_t n, const int32_t *stream_ids, const int32_t *lens,
                       const float *q_dev, float *out_dev, void *stream);

/* qkv_prefill_attend with the queries already in the tensor-core kernel's
 * operand form, as the fused append writes them for prompt rows: q16_dev
 * [sum lens][Hq*D] = q x log2(e) / sqrt(D) rounded to bf16 (bf16 cache) or f16
 * (e4m3 cache).  Saves the f32 -> 16-bit pass over q.  QKV_ERR_STATE for an
 * f32 cache or with the CUDA-core prefill kernel selected. */
int qkv_prefill_attend_q16(qkv_handle *h, int32_t layer, int32_t n, const int32_t *stream_ids, const int32_t *lens,
                           const void *q16_dev, float *out_dev, void *stream);

/* One KV-cache step of the microbench: for each of the n streams append one
 * token and attend, for every layer.  qkv[n_layers][n][Hq*D+2*Hkv*D] f32,
 * out[n_layers][n][Hq*D] f32 (layer-major), device pointers; the streams'
 * lengths grow by 1.  stream_ids is a host array.  Since every layer's
 * projections are given up front, the attention launch of layer l also
 * appends layer l + 1's token (the stored bytes are those of the separate
 * append); a steady batch replays as one CUDA graph. */
int qkv_kv_step(qkv_handle *h, int32_t n, const int32_t *stream_ids, const float *qkv_dev,
                float *out_dev, void *stream);

/* qkv_kv_step with pinned-or-pageable HOST qkv/out buffers: the copies in and
 * out are part of the call (synchronising), pipelined by layer under the
 * kernels (each layer's inputs go up a few layers ahead of their use, its
 * outputs come back as soon as its attention has run).  Pinned buffers
 * replay copies and kernels as one captured graph per (n, buffers). */
int qkv_kv_step_host(qkv_handle *h, int32_t n, const int32_t *stream_ids, const float *qkv_host,
                     float *out_host);

/* Grow an open stream's length by `tokens` without writing K/V (pages are
 * allocated; their contents are whatever the pool holds).  For benches that
 * need long contexts quickly. */
int qkv_stream_extend(qkv_handle *h, int32_t stream_id, int32_t tokens);

/* Fill every page currently owned by open streams, in every layer, with
 * seeded N(0,1) values in the cache dtype (8-bit caches: per-page scales set). */
int qkv_fill_random(qkv_handle *h, uint64_t seed);

/* Page gather: copy tokens [0, len) of one stream's layer cache to host as
 * contiguous k[len][Hkv*D] and v[len][Hkv*D] in the cache dtype (8-bit
 * caches: the raw bytes, e4m3 or excess-128 int8; scales via
 * scales_out[n_pages][2][Hkv][16] when non-NULL). */
int qkv_gather(qkv_handle *h, int32_t layer, int32_t stream_id, void *k_host, void *v_host,
               float *scales_out);

/* Page table of a stream: up to cap page ids into pages_out; *n = pages used. */
int qkv_stream_pages(const qkv_handle *h, int32_t stream_id, int32_t *pages_out, int32_t cap,
                     int32_t *n);

/* Measurement probe, no counterpart in the reference: the HBM read ceiling of
 * the decode-attention kernel's access pattern.  Streams the pages
 * pages_dev[0..n) (device int32 page ids of one layer's pool, in the order the
 * decode attention reads them: each row's pages in turn) into shared memory
 * with the same persistent grid, page split and one bulk copy per page as the
 * decode-attention kernel, and discards them.  bf16 and 8-bit caches (pages of
 * at most 64 KB); asynchronous on `stream` (NULL = the CUDA legacy default
 * stream, as for the other operator-level calls). */
int qkv_page_read_probe(qkv_handle *h, int32_t layer, int32_t n, const int32_t *pages_dev, void *stream);

/* Debug probe of the greedy head (the reference keeps the equivalent hidden
 * row inside text-decoder.cpp:476-493): copies the f32 residual rows [n][H]
 * that the last qkv_decode_step fed to the final RMSNorm and the LM head, in
 * that call's stream order, so a checker can recompute the f32 logits and
 * their argmax (with bf16 weights the device re-scores in f32 every token
 * that could be the f32 argmax; QWENASR_B200_EXACT_ARGMAX=0 turns that off). */
int qkv_debug_residual(qkv_handle *h, int32_t n, float *out);

/* Test of the failure path of the kernels' bounded waits (the reference has
 * no device code; its counterpart is the status checking of
 * text-decoder.cpp:1740-1746).  Launches, on the handle's stream, one CTA that
 * runs the kernels' own bounded waits (the decode-attention stage and
 * hand-over waits, the mbarrier wait of the GEMM and prefill attention) on
 * events nothing completes, each giving up after limit_cycles SM clock cycles
 * (1 .. 4e9, the kernels' own limit) and recording a "bounded wait ran out"
 * device error.  Returns QKV_OK once launched; the next qkv_sync reports
 * QKV_ERR_DEVICE and clears the error, and the handle stays usable. */
int qkv_debug_wait_timeout(qkv_handle *h, int64_t limit_cycles);

/* Synchronise the device and surface any device error. */
int qkv_sync(qkv_handle *h);

/* Device scratch / launch accounting of the last call (for benches). */
int qkv_last_launches(const qkv_handle *h, int64_t *kernels);

/* K2 decode attention for callers that may not allocate device memory: code
 * embedded in a host framework that owns every device buffer through its own
 * allocator and memory plan (a graph scheduler with pre-sized buffers, a
 * server that budgets HBM up front), where a cudaMalloc or cudaFree behind the
 * framework's back breaks its accounting or is not allowed.  This entry point
 * has no counterpart in the reference.  The caller passes everything as device
 * pointers: one layer's pool ([n_pages][2][8][16][128] elements of kv_dtype),
 * its 8-bit scales ([n_pages][2][8][16] f32, or NULL unless kv_dtype is one
 * of the 8-bit caches), the
 * page table [max_streams][maxp], and per-row slots, lengths (tokens to
 * attend over), queries [n][2048] f32 and outputs [n][2048] f32.  No call
 * allocates: the kernel's scratch is a fixed ~3.5 MB array inside this
 * library, which every GPU that loads the library holds until the process
 * exits, and a call takes at most 256 rows (QKV_ERR_CAPACITY beyond).  The
 * first call on each device, with that device current, looks up the array's
 * device address and prepares the kernel; make that first call before any
 * stream capture.  All calls share the one array, which keeps the last call's
 * contents, so calls that overlap on the GPU (two streams, two host threads)
 * race.  The call is asynchronous on `stream` (NULL = legacy default stream)
 * and its status covers the argument checks and the launch only: device-side
 * errors are not reported.  A row that fails the kernel's bounds checks (a
 * slot, length or page id out of range), and any row left when one of the
 * kernel's bounded waits runs out (~2 s), keeps whatever its output held
 * before the call; fill the output with NaN first where that must be seen.
 * err (nullable) receives a message for a non-zero status. */
int qkv_kv_attend_noalloc(const void *pool_layer, int32_t kv_dtype, const float *scales_layer,
                          const int32_t *page_table, int32_t maxp, int32_t max_streams, int32_t n_pages,
                          int32_t n, const int32_t *slots_dev, const int32_t *lens_dev, const float *q_dev,
                          float *out_dev, void *stream, char *err, size_t err_len);

/* Host-only GGUF probe (no GPU): shape / type of one tensor, and up to
 * cap_bytes of its raw data copied to data_out (nullable).  ne_out[4] gets
 * GGML ne (unused dims 1).  The loader checks of gguf-model.cpp:110-162 apply. */
int qkv_gguf_tensor(const char *gguf_path, const char *name, int64_t *ne_out, int32_t *n_dims, int32_t *ggml_type,
                    void *data_out, size_t cap_bytes, char *err, size_t err_len);

/* ---- host-only tokenizer: ASR prompt ids and detokenisation (no GPU) ----
 * The step after the greedy loop: qwenasr_tokenizer_decode (src/tokenizer.cpp:
 * 482-527).  qkv_tokenizer_open reads the byte-level BPE vocabulary and the
 * seven special-token ids from a model file's metadata (the keys and checks
 * of qwenasr_tokenizer_load_gguf, :306-372; QKV_ERR_FORMAT with the
 * reference's message when incomplete).  qkv_tokenizer_decode writes the bytes
 * of ids[0..n) (out-of-range ids skipped; the special tokens too when
 * skip_special) to out, *len = their count; QKV_ERR_CAPACITY when they do not
 * fit in cap (*len still tells how many).  A malformed token whose last UTF-8
 * sequence is cut short yields that sequence followed by zero bytes, as the
 * reference's read runs on into the token's terminator.  Every tokenizer
 * entry returns QKV_ERR_HOST_MEMORY when its tables or output do not fit in
 * host memory. */
int qkv_tokenizer_open(const char *gguf_path, qkv_tokenizer **out, char *err, size_t err_len);
int qkv_tokenizer_decode(const qkv_tokenizer *t, const int32_t *ids, int32_t n, int32_t skip_special, char *out,
                         size_t cap, size_t *len);
/* Encoding, as qwenasr_tokenizer_encode (src/tokenizer.cpp:438-480): the ids
 * of text[0..text_len) (plus the end-of-sequence id when add_eos) into
 * ids[0..cap), *n = their count (QKV_ERR_CAPACITY when more than cap; *n
 * still tells how many).  qkv_asr_prompt_ids encodes the ASR prompt of
 * qwenasr_build_asr_prompt (:529-549): system text, audio_tokens audio
 * placeholders, and the language line when language is non-empty; its ids go
 * to qkv_prefill_ids together with the audio rows.  As in the reference, a
 * UTF-8 sequence cut off at the end of a segment (the text's end, or just
 * before a special token) is read to its announced length: the missing
 * bytes encode as zero bytes. */
int qkv_tokenizer_encode(const qkv_tokenizer *t, const char *text, size_t text_len, int32_t add_eos, int32_t *ids,
                         size_t cap, size_t *n);
int qkv_asr_prompt_ids(const qkv_tokenizer *t, int32_t audio_tokens, const char *system_text, const char *language,
                       int32_t *ids, size_t cap, size_t *n);
void qkv_tokenizer_close(qkv_tokenizer *t);

/* ---- host-only page allocator (no GPU needed; used inside every handle) ----
 * Pages hold page_tokens tokens of every layer's K and V for one stream.
 * qkv_pager_create returns NULL on a bad argument (n_pages outside 1..2^30)
 * or when its free list does not fit in host memory. */
qkv_pager *qkv_pager_create(int64_t n_pages, int32_t page_tokens, int32_t max_streams,
                            int32_t max_pages_per_stream, uint32_t seed);
void qkv_pager_destroy(qkv_pager *p);
int qkv_pager_open(qkv_pager *p, int32_t *stream_id);
int qkv_pager_close(qkv_pager *p, int32_t stream_id);
/* Reserve room for `tokens` more tokens; *new_pages = pages added. */
int qkv_pager_append(qkv_pager *p, int32_t stream_id, int32_t tokens, int32_t *new_pages);
int qkv_pager_length(const qkv_pager *p, int32_t stream_id, int32_t *tokens);
int qkv_pager_pages(const qkv_pager *p, int32_t stream_id, int32_t *pages_out, int32_t cap,
                    int32_t *n);
int64_t qkv_pager_free_pages(const qkv_pager *p);
/* Plan a compaction: live pages above the live count move down into free
 * slots.  Writes up to cap (src, dst) pairs and rewrites the page lists. */
int qkv_pager_compact(qkv_pager *p, int32_t *src, int32_t *dst, int64_t cap, int64_t *n_moves);
/* Consistency check (every page owned once, free list disjoint): 0 if sound. */
int qkv_pager_check(const qkv_pager *p);

#ifdef __cplusplus
}
#endif
#endif
