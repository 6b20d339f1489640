/*
 * qkv_oracle.c -- CPU restatement of the reference's scalar text-decoder path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the thing measured or shipped).
 * Built by oracle/Makefile with -O2 -ffp-contract=off and no -march flag so
 * that, like the reference built with default g++ flags on x86-64, no
 * multiply-add is fused and every float operation rounds on its own.
 *
 * Line citations are to src/text-decoder.cpp of qwenasr.cpp.
 */
#include "qkv_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* :542-557 -- mean square accumulated in double, scale in float,
 * output = (input * scale) * weight. */
void oracle_rms_norm_row(const float *input, int size, const float *weight, float eps, float *output) {
    double mean_square = 0.0;
    for (int i = 0; i < size; ++i) {
        mean_square += (double)input[i] * input[i];
    }
    mean_square /= (double)size;
    const float scale = 1.0f / sqrtf((float)mean_square + eps);
    for (int i = 0; i < size; ++i) {
        output[i] = input[i] * scale * weight[i];
    }
}

/* :559-580 -- rows x W[out][in], float accumulation in input order. */
static void linear(const float *input, int rows, int in_dim, int out_dim, const float *w, float *output) {
    for (int row = 0; row < rows; ++row) {
        const float *src = input + (size_t)row * in_dim;
        float *dst = output + (size_t)row * out_dim;
        for (int o = 0; o < out_dim; ++o) {
            float sum = 0.0f;
            const float *ww = w + (size_t)o * in_dim;
            for (int i = 0; i < in_dim; ++i) {
                sum += src[i] * ww[i];
            }
            dst[o] = sum;
        }
    }
}

/* :600-602 */
float oracle_silu(float x) {
    return x / (1.0f + expf(-x));
}

/* :610-616 -- inv_freq = exp(-log(theta) * 2i / D) in double, angle in double,
 * rounded to float once. */
void oracle_rope_cos_sin(int position, int i, int head_dim, float rope_theta, float *c, float *s) {
    const double log_theta = log((double)rope_theta);
    const double inv_freq = exp(-log_theta * (double)(2 * i) / (double)head_dim);
    const double angle = (double)position * inv_freq;
    *c = (float)cos(angle);
    *s = (float)sin(angle);
}

/* :604-625 -- NEOX rotate-half pairs (i, i + D/2). */
void oracle_rope_position(float *rows, int position, int n_heads, int head_dim, float rope_theta) {
    const int half = head_dim / 2;
    for (int i = 0; i < half; ++i) {
        float c, s;
        oracle_rope_cos_sin(position, i, head_dim, rope_theta, &c, &s);
        for (int head = 0; head < n_heads; ++head) {
            float *row = rows + (size_t)head * head_dim;
            const float a = row[i];
            const float b = row[half + i];
            row[i] = a * c - b * s;
            row[half + i] = b * c + a * s;
        }
    }
}

static void head_norm_inplace(float *x, int n_heads, int head_dim, const float *w, float eps, float *tmp) {
    for (int head = 0; head < n_heads; ++head) {
        float *ptr = x + (size_t)head * head_dim;
        oracle_rms_norm_row(ptr, head_dim, w, eps, tmp);
        memcpy(ptr, tmp, (size_t)head_dim * sizeof(float));
    }
}

/* :643-809 */
int oracle_layer_prefill(const oracle_model *m, int layer, const float *x, int tokens,
                         float *out, float *k_out, float *v_out) {
    const int H = m->hidden, D = m->head_dim, F = m->intermediate;
    const int q_dim = m->n_heads * D, kv_dim = m->n_kv_heads * D;
    if (tokens <= 0 || layer < 0 || layer >= m->n_layers || m->n_heads % m->n_kv_heads != 0) {
        return -1;
    }
    const oracle_layer *t = &m->layers[layer];
    float *normed = (float *)malloc(sizeof(float) * (size_t)tokens * H);
    float *q = (float *)malloc(sizeof(float) * (size_t)tokens * q_dim);
    float *k = (float *)malloc(sizeof(float) * (size_t)tokens * kv_dim);
    float *v = (float *)malloc(sizeof(float) * (size_t)tokens * kv_dim);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)D);
    float *attn = (float *)calloc((size_t)tokens * q_dim, sizeof(float));
    float *scores = (float *)malloc(sizeof(float) * (size_t)tokens);
    float *proj = (float *)malloc(sizeof(float) * (size_t)tokens * H);
    float *hs = (float *)malloc(sizeof(float) * (size_t)tokens * H);
    float *gate = (float *)malloc(sizeof(float) * (size_t)tokens * F);
    float *up = (float *)malloc(sizeof(float) * (size_t)tokens * F);
    float *down = (float *)malloc(sizeof(float) * (size_t)tokens * H);

    for (int tok = 0; tok < tokens; ++tok) {
        oracle_rms_norm_row(x + (size_t)tok * H, H, t->attn_norm, m->rms_norm_eps, normed + (size_t)tok * H);
    }
    linear(normed, tokens, H, q_dim, t->q_w, q);
    linear(normed, tokens, H, kv_dim, t->k_w, k);
    linear(normed, tokens, H, kv_dim, t->v_w, v);
    /* :721-734 per-head QK-norm, q heads then k heads, token by token */
    for (int tok = 0; tok < tokens; ++tok) {
        head_norm_inplace(q + (size_t)tok * q_dim, m->n_heads, D, t->q_norm, m->rms_norm_eps, tmp);
        head_norm_inplace(k + (size_t)tok * kv_dim, m->n_kv_heads, D, t->k_norm, m->rms_norm_eps, tmp);
    }
    /* :736-737 RoPE at positions 0..T-1 */
    for (int tok = 0; tok < tokens; ++tok) {
        oracle_rope_position(q + (size_t)tok * q_dim, tok, m->n_heads, D, m->rope_theta);
    }
    for (int tok = 0; tok < tokens; ++tok) {
        oracle_rope_position(k + (size_t)tok * kv_dim, tok, m->n_kv_heads, D, m->rope_theta);
    }

    /* :739-791 causal GQA attention */
    const int n_rep = m->n_heads / m->n_kv_heads;
    const float scale = 1.0f / sqrtf((float)D);
    for (int tok = 0; tok < tokens; ++tok) {
        for (int head = 0; head < m->n_heads; ++head) {
            const int kvh = head / n_rep;
            const float *qrow = q + (size_t)tok * q_dim + (size_t)head * D;
            float max_score = -INFINITY;
            for (int kt = 0; kt <= tok; ++kt) {
                const float *krow = k + (size_t)kt * kv_dim + (size_t)kvh * D;
                float score = 0.0f;
                for (int d = 0; d < D; ++d) {
                    score += qrow[d] * krow[d];
                }
                score *= scale;
                scores[kt] = score;
                max_score = (max_score < score) ? score : max_score; /* std::max */
            }
            float denom = 0.0f;
            for (int kt = 0; kt <= tok; ++kt) {
                const float value = expf(scores[kt] - max_score);
                scores[kt] = value;
                denom += value;
            }
            float *dst = attn + (size_t)tok * q_dim + (size_t)head * D;
            for (int d = 0; d < D; ++d) {
                float sum = 0.0f;
                for (int kt = 0; kt <= tok; ++kt) {
                    const float prob = scores[kt] / denom;
                    const float *vrow = v + (size_t)kt * kv_dim + (size_t)kvh * D;
                    sum += prob * vrow[d];
                }
                dst[d] = sum;
            }
        }
    }

    linear(attn, tokens, q_dim, H, t->o_w, proj);
    if (k_out) memcpy(k_out, k, sizeof(float) * (size_t)tokens * kv_dim);
    if (v_out) memcpy(v_out, v, sizeof(float) * (size_t)tokens * kv_dim);

    for (size_t i = 0; i < (size_t)tokens * H; ++i) {
        hs[i] = x[i] + proj[i];
    }
    for (int tok = 0; tok < tokens; ++tok) {
        oracle_rms_norm_row(hs + (size_t)tok * H, H, t->ffn_norm, m->rms_norm_eps, normed + (size_t)tok * H);
    }
    linear(normed, tokens, H, F, t->gate_w, gate);
    linear(normed, tokens, H, F, t->up_w, up);
    for (size_t i = 0; i < (size_t)tokens * F; ++i) {
        gate[i] = oracle_silu(gate[i]) * up[i];
    }
    linear(gate, tokens, F, H, t->down_w, down);
    for (size_t i = 0; i < (size_t)tokens * H; ++i) {
        hs[i] += down[i];
    }
    memcpy(out, hs, sizeof(float) * (size_t)tokens * H);

    free(normed); free(q); free(k); free(v); free(tmp); free(attn); free(scores);
    free(proj); free(hs); free(gate); free(up); free(down);
    return 0;
}

/* :1000-1024 -- QK-norm then RoPE at `position`; V stays raw. */
void oracle_append_qkv(const float *qkv_raw, const float *q_norm_w, const float *k_norm_w,
                       int position, int n_heads, int n_kv_heads, int head_dim,
                       float rope_theta, float eps, float *q_out, float *k_out, float *v_out) {
    const int q_dim = n_heads * head_dim, kv_dim = n_kv_heads * head_dim;
    float tmp[1024];
    memcpy(q_out, qkv_raw, sizeof(float) * (size_t)q_dim);
    memcpy(k_out, qkv_raw + q_dim, sizeof(float) * (size_t)kv_dim);
    memcpy(v_out, qkv_raw + q_dim + kv_dim, sizeof(float) * (size_t)kv_dim);
    head_norm_inplace(q_out, n_heads, head_dim, q_norm_w, eps, tmp);
    head_norm_inplace(k_out, n_kv_heads, head_dim, k_norm_w, eps, tmp);
    oracle_rope_position(q_out, position, n_heads, head_dim, rope_theta);
    oracle_rope_position(k_out, position, n_kv_heads, head_dim, rope_theta);
}

/* :1029-1075 */
void oracle_attend(const float *q, const float *k_cache, const float *v_cache, int tokens,
                   int n_heads, int n_kv_heads, int head_dim, float *out) {
    const int kv_dim = n_kv_heads * head_dim;
    const int n_rep = n_heads / n_kv_heads;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float *scores = (float *)malloc(sizeof(float) * (size_t)tokens);
    for (int head = 0; head < n_heads; ++head) {
        const int kvh = head / n_rep;
        const float *qrow = q + (size_t)head * head_dim;
        float max_score = -INFINITY;
        for (int kt = 0; kt < tokens; ++kt) {
            const float *krow = k_cache + (size_t)kt * kv_dim + (size_t)kvh * head_dim;
            float score = 0.0f;
            for (int d = 0; d < head_dim; ++d) {
                score += qrow[d] * krow[d];
            }
            score *= scale;
            scores[kt] = score;
            max_score = (max_score < score) ? score : max_score; /* std::max */
        }
        float denom = 0.0f;
        for (int kt = 0; kt < tokens; ++kt) {
            const float value = expf(scores[kt] - max_score);
            scores[kt] = value;
            denom += value;
        }
        float *dst = out + (size_t)head * head_dim;
        for (int d = 0; d < head_dim; ++d) {
            float sum = 0.0f;
            for (int kt = 0; kt < tokens; ++kt) {
                const float prob = scores[kt] / denom;
                const float *vrow = v_cache + (size_t)kt * kv_dim + (size_t)kvh * head_dim;
                sum += prob * vrow[d];
            }
            dst[d] = sum;
        }
    }
    free(scores);
}

/* :958-1098 */
int oracle_layer_decode(const oracle_model *m, int layer, const float *x, float *k_cache,
                        float *v_cache, int capacity, int *cache_tokens, float *out) {
    const int H = m->hidden, D = m->head_dim, F = m->intermediate;
    const int q_dim = m->n_heads * D, kv_dim = m->n_kv_heads * D;
    if (*cache_tokens <= 0 || *cache_tokens >= capacity || layer < 0 || layer >= m->n_layers) {
        return -1;
    }
    const oracle_layer *t = &m->layers[layer];
    float *normed = (float *)malloc(sizeof(float) * (size_t)H);
    float *qkv = (float *)malloc(sizeof(float) * (size_t)(q_dim + 2 * kv_dim));
    float *q = (float *)malloc(sizeof(float) * (size_t)q_dim);
    float *attn = (float *)malloc(sizeof(float) * (size_t)q_dim);
    float *proj = (float *)malloc(sizeof(float) * (size_t)H);
    float *hs = (float *)malloc(sizeof(float) * (size_t)H);
    float *gate = (float *)malloc(sizeof(float) * (size_t)F);
    float *up = (float *)malloc(sizeof(float) * (size_t)F);
    float *down = (float *)malloc(sizeof(float) * (size_t)H);

    oracle_rms_norm_row(x, H, t->attn_norm, m->rms_norm_eps, normed);
    linear(normed, 1, H, q_dim, t->q_w, qkv);
    linear(normed, 1, H, kv_dim, t->k_w, qkv + q_dim);
    linear(normed, 1, H, kv_dim, t->v_w, qkv + q_dim + kv_dim);

    const int position = *cache_tokens;
    oracle_append_qkv(qkv, t->q_norm, t->k_norm, position, m->n_heads, m->n_kv_heads, D,
                      m->rope_theta, m->rms_norm_eps, q,
                      k_cache + (size_t)position * kv_dim, v_cache + (size_t)position * kv_dim);
    *cache_tokens = position + 1;
    oracle_attend(q, k_cache, v_cache, *cache_tokens, m->n_heads, m->n_kv_heads, D, attn);

    linear(attn, 1, q_dim, H, t->o_w, proj);
    for (int i = 0; i < H; ++i) hs[i] = x[i] + proj[i];
    oracle_rms_norm_row(hs, H, t->ffn_norm, m->rms_norm_eps, normed);
    linear(normed, 1, H, F, t->gate_w, gate);
    linear(normed, 1, H, F, t->up_w, up);
    for (int i = 0; i < F; ++i) gate[i] = oracle_silu(gate[i]) * up[i];
    linear(gate, 1, F, H, t->down_w, down);
    for (int i = 0; i < H; ++i) hs[i] += down[i];
    memcpy(out, hs, sizeof(float) * (size_t)H);

    free(normed); free(qkv); free(q); free(attn); free(proj); free(hs); free(gate); free(up); free(down);
    return 0;
}

/* :910-956 */
void oracle_logits(const oracle_model *m, const float *state, float *logits) {
    const int H = m->hidden;
    float *normed = (float *)malloc(sizeof(float) * (size_t)H);
    oracle_rms_norm_row(state, H, m->output_norm, m->rms_norm_eps, normed);
    for (int tok = 0; tok < m->vocab; ++tok) {
        const float *ww = m->output_w + (size_t)tok * H;
        float sum = 0.0f;
        for (int i = 0; i < H; ++i) {
            sum += normed[i] * ww[i];
        }
        logits[tok] = sum;
    }
    free(normed);
}

/* :2136-2144 */
int32_t oracle_argmax(const float *logits, int vocab) {
    int32_t next_id = -1;
    float best = -INFINITY;
    for (int i = 0; i < vocab; ++i) {
        if (logits[i] > best) {
            best = logits[i];
            next_id = i;
        }
    }
    return next_id;
}

/* :1856-1925 */
int oracle_prefill_logits(const oracle_model *m, const float *x, int tokens, float *logits) {
    const size_t n = (size_t)tokens * m->hidden;
    float *a = (float *)malloc(sizeof(float) * n);
    float *b = (float *)malloc(sizeof(float) * n);
    memcpy(a, x, sizeof(float) * n);
    for (int layer = 0; layer < m->n_layers; ++layer) {
        if (oracle_layer_prefill(m, layer, a, tokens, b, NULL, NULL) != 0) {
            free(a); free(b);
            return -1;
        }
        float *t = a; a = b; b = t;
    }
    oracle_logits(m, a + (size_t)(tokens - 1) * m->hidden, logits);
    free(a); free(b);
    return 0;
}

/* Shared body of the cached greedy loop (:2033-2207).  forced_ids == NULL runs
 * the reference loop; otherwise the decoded id of step s is forced_ids[s]. */
static int generate_impl(const oracle_model *m, const float *x, int tokens, int max_new_tokens,
                         const int32_t *stop_ids, int n_stop, const int32_t *forced_ids,
                         int32_t *out_ids, int *n_out, int *stopped, float *step_logits,
                         float *k_dump, float *v_dump) {
    const int H = m->hidden, L = m->n_layers, V = m->vocab;
    const int kv_dim = m->n_kv_heads * m->head_dim;
    const int cap = tokens + max_new_tokens;
    if (n_out) *n_out = 0;
    if (stopped) *stopped = 0;
    if (max_new_tokens <= 0) return max_new_tokens < 0 ? -1 : 0;

    float *kc = (float *)malloc(sizeof(float) * (size_t)L * cap * kv_dim);
    float *vc = (float *)malloc(sizeof(float) * (size_t)L * cap * kv_dim);
    int *lens = (int *)calloc((size_t)L, sizeof(int));
    float *a = (float *)malloc(sizeof(float) * (size_t)tokens * H);
    float *b = (float *)malloc(sizeof(float) * (size_t)tokens * H);
    float *logits = (float *)malloc(sizeof(float) * (size_t)V);
    int rc = 0;

    memcpy(a, x, sizeof(float) * (size_t)tokens * H);
    for (int layer = 0; layer < L; ++layer) {
        if (oracle_layer_prefill(m, layer, a, tokens, b, kc + (size_t)layer * cap * kv_dim,
                                 vc + (size_t)layer * cap * kv_dim) != 0) {
            rc = -1;
            goto done;
        }
        lens[layer] = tokens;
        float *t = a; a = b; b = t;
    }
    oracle_logits(m, a + (size_t)(tokens - 1) * H, logits);

    for (int step = 0; step < max_new_tokens; ++step) {
        const int32_t next_id = oracle_argmax(logits, V);
        if (next_id < 0 || next_id >= V) {
            rc = -2;
            goto done;
        }
        if (step_logits) memcpy(step_logits + (size_t)step * V, logits, sizeof(float) * (size_t)V);
        out_ids[step] = next_id;
        if (n_out) *n_out = step + 1;
        int stop = 0;
        for (int i = 0; i < n_stop; ++i) {
            if (next_id == stop_ids[i]) { stop = 1; break; }
        }
        if (stop && !forced_ids) {
            if (stopped) *stopped = 1;
            break;
        }
        if (step + 1 >= max_new_tokens) break;

        const int32_t fed = forced_ids ? forced_ids[step] : next_id;
        memcpy(a, m->embd + (size_t)fed * H, sizeof(float) * (size_t)H);
        for (int layer = 0; layer < L; ++layer) {
            if (oracle_layer_decode(m, layer, a, kc + (size_t)layer * cap * kv_dim,
                                    vc + (size_t)layer * cap * kv_dim, cap, &lens[layer], b) != 0) {
                rc = -1;
                goto done;
            }
            float *t = a; a = b; b = t;
        }
        oracle_logits(m, a, logits);
    }
    if (k_dump) memcpy(k_dump, kc, sizeof(float) * (size_t)L * cap * kv_dim);
    if (v_dump) memcpy(v_dump, vc, sizeof(float) * (size_t)L * cap * kv_dim);
done:
    free(kc); free(vc); free(lens); free(a); free(b); free(logits);
    return rc;
}

int oracle_generate_cached(const oracle_model *m, const float *x, int tokens, int max_new_tokens,
                           const int32_t *stop_ids, int n_stop, int32_t *out_ids, int *n_out,
                           int *stopped, float *step_logits, float *k_dump, float *v_dump) {
    return generate_impl(m, x, tokens, max_new_tokens, stop_ids, n_stop, NULL, out_ids, n_out,
                         stopped, step_logits, k_dump, v_dump);
}

int oracle_generate_forced(const oracle_model *m, const float *x, int tokens, int n_steps,
                           const int32_t *forced_ids, int32_t *argmax_ids, float *step_logits) {
    int n_out = 0, stopped = 0;
    return generate_impl(m, x, tokens, n_steps, NULL, 0, forced_ids, argmax_ids, &n_out, &stopped,
                         step_logits, NULL, NULL);
}

int oracle_kv_step_batch(int n_streams, int n_layers, const float *qkv, const float *q_norm_w,
                         const float *k_norm_w, float *const *k_caches, float *const *v_caches,
                         const int *capacity, int *lens, int n_heads, int n_kv_heads, int head_dim,
                         float rope_theta, float eps, float *out, int n_threads) {
    const int q_dim = n_heads * head_dim, kv_dim = n_kv_heads * head_dim;
    const int row = q_dim + 2 * kv_dim;
    int bad = 0;
    for (int s = 0; s < n_streams; ++s) {
        if (lens[s] < 0 || lens[s] >= capacity[s]) bad = 1;
    }
    if (bad) return -1;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int s = 0; s < n_streams; ++s) {
        float q[4096];
        const int pos = lens[s];
        for (int layer = 0; layer < n_layers; ++layer) {
            float *kc = k_caches[s] + (size_t)layer * capacity[s] * kv_dim;
            float *vc = v_caches[s] + (size_t)layer * capacity[s] * kv_dim;
            oracle_append_qkv(qkv + ((size_t)layer * n_streams + s) * row,
                              q_norm_w + (size_t)layer * head_dim, k_norm_w + (size_t)layer * head_dim, pos,
                              n_heads, n_kv_heads, head_dim, rope_theta, eps, q,
                              kc + (size_t)pos * kv_dim, vc + (size_t)pos * kv_dim);
            oracle_attend(q, kc, vc, pos + 1, n_heads, n_kv_heads, head_dim,
                          out + ((size_t)layer * n_streams + s) * q_dim);
        }
        lens[s] = pos + 1;
    }
    (void)n_threads;
    return 0;
}

/* src/decoder-input.cpp:64-98 (qwenasr_decoder_input_from_audio, after the
 * prompt is tokenised): embedding copy, then the audio row over it. */
int oracle_decoder_input(const int32_t *ids, int tokens, const float *embd, int vocab, int hidden,
                         const float *audio, int audio_tokens, int32_t audio_token_id, float *out) {
    int audio_positions = 0;
    for (int t = 0; t < tokens; ++t) {
        const int32_t id = ids[t];
        if (id < 0 || id >= vocab) return 1;
        float *dst = out + (size_t)t * hidden;
        memcpy(dst, embd + (size_t)id * hidden, (size_t)hidden * sizeof(float));
        if (id == audio_token_id) {
            if (audio_positions >= audio_tokens) return 2;
            memcpy(dst, audio + (size_t)audio_positions * hidden, (size_t)hidden * sizeof(float));
            ++audio_positions;
        }
    }
    return audio_positions == audio_tokens ? 0 : 3;
}
