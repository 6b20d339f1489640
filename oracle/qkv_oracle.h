/*
 * qkv_oracle.h -- CPU restatement of the Qwen3-ASR text decoder's scalar
 * KV-cache path (reference: src/text-decoder.cpp of qwenasr.cpp).
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is
 * compared against. It is loaded by tests/, by __graft_entry__.smoke() and by
 * the cpu_baseline / --impl reference legs of bench.py, and by nothing else.
 * The product library never links or calls it.
 *
 * Every function follows the reference's loop order and accumulation types
 * (float dot products accumulated left to right, RMSNorm mean-square in
 * double, RoPE angle in double), so that on the same inputs it reproduces the
 * reference's scalar arithmetic bit for bit.  The pin is checked by
 * tests/test_oracle.py against fixtures produced by the reference's own scalar
 * code (oracle/_ref) and by its PyTorch restatement (the benchmarks/check_text_* scripts).
 *
 * Weight layout: GGML ne = [in, out], i.e. row-major W[out][in].
 */
#ifndef QKV_ORACLE_H
#define QKV_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct oracle_layer {
    const float *attn_norm;  /* [H]            text.blk.N.attn_norm.weight */
    const float *ffn_norm;   /* [H]            text.blk.N.ffn_norm.weight */
    const float *q_w;        /* [Hq*D][H]      text.blk.N.attn_q.weight */
    const float *k_w;        /* [Hkv*D][H]     text.blk.N.attn_k.weight */
    const float *v_w;        /* [Hkv*D][H]     text.blk.N.attn_v.weight */
    const float *o_w;        /* [H][Hq*D]      text.blk.N.attn_output.weight */
    const float *q_norm;     /* [D]            text.blk.N.attn_q_norm.weight */
    const float *k_norm;     /* [D]            text.blk.N.attn_k_norm.weight */
    const float *gate_w;     /* [F][H]         text.blk.N.ffn_gate.weight */
    const float *up_w;       /* [F][H]         text.blk.N.ffn_up.weight */
    const float *down_w;     /* [H][F]         text.blk.N.ffn_down.weight */
} oracle_layer;

typedef struct oracle_model {
    int n_layers, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab;
    float rope_theta, rms_norm_eps;
    const oracle_layer *layers;   /* n_layers entries */
    const float *embd;            /* [V][H] text.token_embd.weight */
    const float *output_norm;     /* [H]    text.output_norm.weight */
    const float *output_w;        /* [V][H] text.output.weight */
} oracle_model;

/* text-decoder.cpp:542-557 */
void oracle_rms_norm_row(const float *input, int size, const float *weight, float eps, float *output);
/* text-decoder.cpp:604-625 (NEOX pairs (i, i+D/2), double angle) */
void oracle_rope_position(float *rows, int position, int n_heads, int head_dim, float rope_theta);
/* The (cos, sin) pair the reference derives for (position, i): text-decoder.cpp:610-616 */
void oracle_rope_cos_sin(int position, int i, int head_dim, float rope_theta, float *c, float *s);
/* text-decoder.cpp:600-602 */
float oracle_silu(float x);

/* One block over T prompt tokens at positions 0..T-1 (text-decoder.cpp:643-809).
 * k_out / v_out (nullable) receive the cached K (post-norm, post-RoPE) and raw V,
 * [T][Hkv*D], exactly what TextLayerKvCache keeps (:771-776). */
int oracle_layer_prefill(const oracle_model *m, int layer, const float *x, int tokens,
                         float *out, float *k_out, float *v_out);

/* One cached decode step of one block (text-decoder.cpp:958-1098).  The cache
 * arrays are [capacity][Hkv*D]; *cache_tokens is the position of the new token
 * and is incremented. */
int oracle_layer_decode(const oracle_model *m, int layer, const float *x, float *k_cache,
                        float *v_cache, int capacity, int *cache_tokens, float *out);

/* Final norm + LM head for one state row (text-decoder.cpp:910-956). */
void oracle_logits(const oracle_model *m, const float *state, float *logits);

/* First-maximum argmax, strict '>' from -inf (text-decoder.cpp:2136-2144). -1 if none. */
int32_t oracle_argmax(const float *logits, int vocab);

/* Full prefill logits of the last prompt row (text-decoder.cpp:1856-1925). */
int oracle_prefill_logits(const oracle_model *m, const float *x, int tokens, float *logits);

/* Greedy generation with a KV cache (text-decoder.cpp:2033-2207).
 * out_ids has room for max_new_tokens ids; *n_out and *stopped are written.
 * step_logits (nullable) receives [max_new_tokens][V]: the logits each id was
 * chosen from.  k_dump/v_dump (nullable) receive the final caches,
 * [n_layers][T+max_new_tokens][Hkv*D]; rows past the final length are left untouched. */
int oracle_generate_cached(const oracle_model *m, const float *x, int tokens, int max_new_tokens,
                           const int32_t *stop_ids, int n_stop, int32_t *out_ids, int *n_out,
                           int *stopped, float *step_logits, float *k_dump, float *v_dump);

/* Teacher-forced variant: decodes the given ids instead of its own argmax and
 * records the argmax and logits of every step, so a device path can be compared
 * step by step on an identical prefix. forced_ids has n_steps-1 entries. */
int oracle_generate_forced(const oracle_model *m, const float *x, int tokens, int n_steps,
                           const int32_t *forced_ids, int32_t *argmax_ids, float *step_logits);

/* The K/V append half of a cached decode step (text-decoder.cpp:1000-1027):
 * qkv_raw = [q(Hq*D) | k(Hkv*D) | v(Hkv*D)] straight out of the projections.
 * Writes q_out (post norm + RoPE), k_out (post norm + RoPE) and v_out (raw). */
void oracle_append_qkv(const float *qkv_raw, const float *q_norm_w, const float *k_norm_w,
                       int position, int n_heads, int n_kv_heads, int head_dim,
                       float rope_theta, float eps, float *q_out, float *k_out, float *v_out);

/* The attention half of a cached decode step (text-decoder.cpp:1029-1075):
 * q [Hq*D], caches [tokens][Hkv*D] -> out [Hq*D]. */
void oracle_attend(const float *q, const float *k_cache, const float *v_cache, int tokens,
                   int n_heads, int n_kv_heads, int head_dim, float *out);

/* Batched microbench leg: for every stream, every layer: append one token
 * (oracle_append_qkv) into its contiguous cache, then attend (oracle_attend).
 * Streams are independent and are spread over n_threads OpenMP threads (the
 * reference itself is single-threaded per stream).
 * qkv: [n_layers][n_streams][Hq*D + 2*Hkv*D] (layer-major, as qkv_kv_step);
 * q_norm_w / k_norm_w: [n_layers][head_dim]; caches: per stream s a pointer to
 * [n_layers][capacity[s]][Hkv*D] for K and for V; lens: tokens already cached
 * (incremented); out: [n_layers][n_streams][Hq*D]. */
/* Decoder input (src/decoder-input.cpp:64-98): row t of out = embedding row
 * ids[t]; a row whose id is audio_token_id takes the next audio row instead
 * (in order).  Checks as the reference does, in its order: 1 = an id outside
 * [0, vocab), 2 = more placeholders than audio rows, 3 = fewer (the counts
 * differ at the end); 0 = ok.  embd [vocab][hidden], audio [audio_tokens][hidden]. */
int oracle_decoder_input(const int32_t *ids, int tokens, const float *embd, int vocab, int hidden,
                         const float *audio, int audio_tokens, int32_t audio_token_id, float *out);

int oracle_kv_step_batch(int n_streams, int n_layers, const float *qkv, const float *q_norm_w,
                         const float *k_norm_w, float *const *k_caches, float *const *v_caches,
                         const int *capacity, int *lens, int n_heads, int n_kv_heads, int head_dim,
                         float rope_theta, float eps, float *out, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
