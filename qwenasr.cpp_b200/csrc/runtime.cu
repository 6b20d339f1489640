// C ABI implementation: handle creation (weights, pool, scratch), the stream
// table, and the prefill / decode / operator-level entry points.
#include "runtime.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <functional>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "gguf.h"

using qkv::DevError;

namespace qkv {

int fail(qkv_handle *h, int code, const std::string &msg) {
    if (h) h->last_error = msg;
    return code;
}

int cuda_fail(qkv_handle *h, cudaError_t e, const char *what) {
    return fail(h, QKV_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// An NVTX range around a C entry point, so a profiler's timeline (and ncu's
// --nvtx filters) can pick out prefill, decode and the operator steps; a
// load and a branch when no tool is attached.
struct TraceRange {
    explicit TraceRange(const char *name) { nvtxRangePushA(name); }
    ~TraceRange() { nvtxRangePop(); }
    TraceRange(const TraceRange &) = delete;
    TraceRange &operator=(const TraceRange &) = delete;
};

// Owner of a temporary device buffer of a host-driven call (the compaction
// move list, the fill list, a gather target): freed on every return path,
// including the early returns of a failed CUDA call.
struct DeviceTemp {
    void *p = nullptr;
    DeviceTemp() = default;
    DeviceTemp(const DeviceTemp &) = delete;
    DeviceTemp &operator=(const DeviceTemp &) = delete;
    ~DeviceTemp() {
        if (p) cudaFree(p);
    }
};

// Handle set-up sizes host tables (the RoPE table, page tables, the pager's
// lists) from the runtime config: a config that passes the checks but does
// not fit in host memory fails with a status instead of an exception
// crossing the C ABI.
template <typename F> int host_alloc_guard(qkv_handle *h, F &&body) {
    try {
        return body();
    } catch (const std::exception &ex) {
        return fail(h, QKV_ERR_HOST_MEMORY, std::string("host allocation failed during set-up: ") + ex.what());
    }
}

}  // namespace qkv

#define CK(call)                                                  \
    do {                                                          \
        cudaError_t e_ = (call);                                  \
        if (e_ != cudaSuccess) return qkv::cuda_fail(h, e_, #call); \
    } while (0)

namespace {

using namespace qkv;

void set_err(char *err, size_t len, const std::string &msg) {
    if (err && len > 0) {
        std::strncpy(err, msg.c_str(), len - 1);
        err[len - 1] = '\0';
    }
}

int validate_model(const qkv_model_config &c, std::string *e) {
    if (c.n_layers <= 0 || c.hidden <= 0 || c.intermediate <= 0 || c.vocab <= 0) {
        *e = "model config: non-positive dimension";
        return QKV_ERR_INVALID_ARG;
    }
    if (c.head_dim != kHeadDim || c.n_heads != kHq || c.n_kv_heads != kHkv) {
        *e = "model config: kernels serve head_dim 128 with 16 q heads and 8 kv heads (got " +
             std::to_string(c.head_dim) + "/" + std::to_string(c.n_heads) + "/" + std::to_string(c.n_kv_heads) + ")";
        return QKV_ERR_INVALID_ARG;
    }
    if (c.hidden % 16 != 0 || c.intermediate % 64 != 0) {
        *e = "model config: hidden must be a multiple of 16 and intermediate a multiple of 64";
        return QKV_ERR_INVALID_ARG;
    }
    if (!(c.rope_theta > 0.0f) || !(c.rms_norm_eps >= 0.0f)) {
        *e = "model config: bad rope_theta or rms_norm_eps";
        return QKV_ERR_INVALID_ARG;
    }
    return QKV_OK;
}

int validate_rt(const qkv_runtime_config &r, std::string *e) {
    if (r.page_tokens != kPageTokens) {
        *e = "runtime config: page_tokens must be 16";
        return QKV_ERR_INVALID_ARG;
    }
    if (r.kv_dtype < QKV_F32 || r.kv_dtype > QKV_E4M3K_I8V ||
        (r.weight_dtype != QKV_F32 && r.weight_dtype != QKV_BF16 && r.weight_dtype != QKV_FP8_E4M3)) {
        *e = "runtime config: bad dtype";
        return QKV_ERR_INVALID_ARG;
    }
    if (r.max_streams <= 0 || r.max_context <= 0 || r.max_pages < 0 || r.max_batch_tokens < 0) {
        *e = "runtime config: bad capacity";
        return QKV_ERR_INVALID_ARG;
    }
    return QKV_OK;
}

// Device, stream, pool, page table, RoPE table, pager, per-step scratch.
int setup_common(qkv_handle *h, bool with_model_scratch) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) return fail(h, QKV_ERR_NO_DEVICE, "no CUDA device");
    if (h->rt.device < 0 || h->rt.device >= ndev) return fail(h, QKV_ERR_NO_DEVICE, "device ordinal out of range");
    h->device = h->rt.device;
    CK(cudaSetDevice(h->device));
    cudaDeviceProp prop{};
    CK(cudaGetDeviceProperties(&prop, h->device));
    if (prop.major != 10) {
        return fail(h, QKV_ERR_NO_DEVICE, std::string("kernels are built for sm_100a; device is ") + prop.name);
    }
    h->num_sms = prop.multiProcessorCount;
    CK(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));

    const qkv_model_config &c = h->cfg;
    h->maxp = (h->rt.max_context + kPageTokens - 1) / kPageTokens;
    const int64_t pages = h->rt.max_pages > 0 ? h->rt.max_pages : static_cast<int64_t>(h->rt.max_streams) * h->maxp;
    if (pages > (int64_t{1} << 30)) return fail(h, QKV_ERR_INVALID_ARG, "max_pages too large");
    h->n_pages = static_cast<int>(pages);
    h->page_bytes = static_cast<size_t>(2) * kPageHalfElems * kv_elem_bytes(h->rt.kv_dtype);
    h->pool_layer_bytes = h->page_bytes * static_cast<size_t>(h->n_pages);
    CK(cudaMalloc(&h->pool, h->pool_layer_bytes * c.n_layers));
    CK(cudaMemsetAsync(h->pool, 0, h->pool_layer_bytes * c.n_layers, h->stream));
    if (kv_is_8bit(h->rt.kv_dtype)) {
        h->scales_layer_elems = static_cast<size_t>(h->n_pages) * kPageScales;
        CK(cudaMalloc(&h->scales, h->scales_layer_elems * c.n_layers * sizeof(float)));
        std::vector<float> ones(h->scales_layer_elems * c.n_layers, 1.0f);
        CK(cudaMemcpy(h->scales, ones.data(), ones.size() * sizeof(float), cudaMemcpyHostToDevice));
    }
    const size_t pt = static_cast<size_t>(h->rt.max_streams) * h->maxp;
    CK(cudaMalloc(&h->d_page_table, pt * sizeof(int)));
    CK(cudaMallocHost(&h->h_page_table, pt * sizeof(int)));
    std::fill(h->h_page_table, h->h_page_table + pt, -1);
    CK(cudaMemcpy(h->d_page_table, h->h_page_table, pt * sizeof(int), cudaMemcpyHostToDevice));

    // RoPE (cos, sin) per (position, i): the reference's double-angle formula
    // (text-decoder.cpp:610-616) evaluated on the host, rounded to float once.
    h->rope_len = h->rt.max_context;
    std::vector<float2> rope(static_cast<size_t>(h->rope_len) * (kHeadDim / 2));
    const double log_theta = std::log(static_cast<double>(c.rope_theta));
    for (int i = 0; i < kHeadDim / 2; ++i) {
        const double inv_freq = std::exp(-log_theta * static_cast<double>(2 * i) / static_cast<double>(kHeadDim));
        for (int pos = 0; pos < h->rope_len; ++pos) {
            const double angle = static_cast<double>(pos) * inv_freq;
            rope[static_cast<size_t>(pos) * (kHeadDim / 2) + i] =
                make_float2(static_cast<float>(std::cos(angle)), static_cast<float>(std::sin(angle)));
        }
    }
    CK(cudaMalloc(&h->d_rope, rope.size() * sizeof(float2)));
    CK(cudaMemcpy(h->d_rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice));

    h->pager = new Pager(h->n_pages, kPageTokens, h->rt.max_streams, h->maxp, h->rt.page_order_seed);
    h->last_id.assign(static_cast<size_t>(h->rt.max_streams), -1);

    const int batch_tokens = h->rt.max_batch_tokens > 0 ? h->rt.max_batch_tokens : h->rt.max_context;
    h->max_rows = std::max(batch_tokens, h->rt.max_streams);
    const size_t R = static_cast<size_t>(h->max_rows);
    const size_t act = h->act_dtype == kActF32 ? 4 : 2;
    CK(cudaMalloc(&h->qkv, R * kQkvDim * sizeof(float)));
    CK(cudaMalloc(&h->q, R * kQDim * sizeof(float)));
    CK(cudaMalloc(&h->q_alt, static_cast<size_t>(h->rt.max_streams) * kQDim * sizeof(float)));
    if (with_model_scratch) {
        CK(cudaMalloc(&h->x, R * c.hidden * sizeof(float)));
        CK(cudaMalloc(&h->xn, R * c.hidden * act));
        CK(cudaMalloc(&h->attn, R * kQDim * act));
        CK(cudaMalloc(&h->gu, R * 2 * c.intermediate * sizeof(float)));
        CK(cudaMalloc(&h->act, R * c.intermediate * act));
        CK(cudaMalloc(&h->qkv_sl, static_cast<size_t>(qkv_handle::kQkvMaxSlices) * h->rt.max_streams * kQkvDim *
                                      sizeof(float)));
        CK(cudaMalloc(&h->res_sl, static_cast<size_t>(qkv_handle::kResMaxSlices) * h->rt.max_streams * c.hidden *
                                      sizeof(float)));
        // stream-K of the fused gate/up GEMM: two token tiles of 2F / 128 weight tiles, 4 parts of 128 x 64 each
        h->sk_flag_tiles = 2 * ((2 * c.intermediate + 127) / 128);
        h->sk_ws_floats = static_cast<size_t>(h->sk_flag_tiles) * 4 * 128 * 64;
        CK(cudaMalloc(&h->sk_ws, h->sk_ws_floats * sizeof(float)));
        CK(cudaMalloc(&h->sk_flags, static_cast<size_t>(h->sk_flag_tiles) * 4 * sizeof(int)));
        CK(cudaMemset(h->sk_flags, 0, static_cast<size_t>(h->sk_flag_tiles) * 4 * sizeof(int)));
        if (h->proj_fp8) {
            CK(cudaMalloc(&h->xq, R * static_cast<size_t>(std::max(c.hidden, std::max(c.intermediate, kQDim)))));
            CK(cudaMalloc(&h->xq_s, R * sizeof(float)));
        }
        CK(cudaMalloc(&h->logits, static_cast<size_t>(h->rt.max_streams) * c.vocab * sizeof(float)));
        const size_t ms = static_cast<size_t>(h->rt.max_streams);
        CK(cudaMalloc(&h->am_v, ms * qkv_handle::kArgmaxSlices * sizeof(float)));
        CK(cudaMalloc(&h->am_i, ms * qkv_handle::kArgmaxSlices * sizeof(int)));
        CK(cudaMalloc(&h->am_cnt, ms * sizeof(int)));
        CK(cudaMemset(h->am_cnt, 0, ms * sizeof(int)));
        CK(cudaMalloc(&h->am_keys, ms * sizeof(unsigned long long)));
        CK(cudaMemset(h->am_keys, 0, ms * sizeof(unsigned long long)));
        CK(cudaMalloc(&h->am_rcnt, ms * sizeof(int)));
        CK(cudaMemset(h->am_rcnt, 0, ms * sizeof(int)));
        CK(cudaMalloc(&h->d_wout_norm, sizeof(float)));
        CK(cudaMemset(h->d_wout_norm, 0, sizeof(float)));
        const char *ea = std::getenv("QWENASR_B200_EXACT_ARGMAX");
        h->exact_argmax = !(ea && std::strcmp(ea, "0") == 0);
    }
    CK(cudaMalloc(&h->d_rowbuf, 4 * R * sizeof(int)));
    CK(cudaMallocHost(&h->h_rowbuf, qkv_handle::kRowRing * 4 * R * sizeof(int)));
    for (auto &ev : h->row_ev) CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&h->items_ev, cudaEventDisableTiming));
    CK(cudaMalloc(&h->d_out_ids, R * sizeof(int)));
    CK(cudaMallocHost(&h->h_out_ids, R * sizeof(int)));
    if (with_model_scratch) {
        CK(cudaMallocHost(&h->h_dec, 2 * R * sizeof(int)));
        CK(cudaMalloc(&h->d_dec, 2 * R * sizeof(int)));
        CK(cudaMallocHost(reinterpret_cast<void **>(&h->h_rowptr), R * sizeof(float *)));
        CK(cudaMalloc(reinterpret_cast<void **>(&h->d_rowptr), R * sizeof(float *)));
        CK(cudaEventCreateWithFlags(&h->dec_ev, cudaEventDisableTiming));
        for (int i = 0; i < qkv_handle::kEmbRing; ++i) {
            CK(cudaMallocHost(&h->h_emb[i], qkv_handle::kEmbChunkBytes));
            CK(cudaEventCreateWithFlags(&h->emb_ev[i], cudaEventDisableTiming));
        }
    }
    h->max_items = (h->max_rows / 64 + h->rt.max_streams + 1) * kHkv;
    CK(cudaMalloc(&h->d_items, static_cast<size_t>(h->max_items) * sizeof(int4)));
    CK(cudaMallocHost(&h->h_items, static_cast<size_t>(h->max_items) * sizeof(int4)));
    const size_t slots = static_cast<size_t>(kAttnMaxRows + h->num_sms);
    CK(cudaMalloc(&h->part_o, slots * kHq * kHeadDim * sizeof(float)));
    CK(cudaMalloc(&h->part_ml, slots * kHq * 2 * sizeof(float)));
    CK(cudaMalloc(&h->counters, static_cast<size_t>(kAttnMaxRows) * kHkv * sizeof(int)));
    CK(cudaMemset(h->counters, 0, static_cast<size_t>(kAttnMaxRows) * kHkv * sizeof(int)));
    CK(cudaMalloc(&h->d_err, sizeof(DevError)));
    CK(cudaMemset(h->d_err, 0, sizeof(DevError)));
    CK(cudaMallocHost(&h->h_err, sizeof(DevError)));
    CK(prepare_decode_attn());
    CK(prepare_gemm_tc());
    CK(prepare_prefill_tc());
    {
        const char *pa = getenv("QWENASR_B200_PREFILL_ATTN");
        h->prefill_tc = !(pa && std::strcmp(pa, "cuda_core") == 0);
        const char *fs = getenv("QWENASR_B200_FUSED_SWIGLU");
        h->fused_swiglu = !(fs && std::strcmp(fs, "0") == 0);
        const char *sk = getenv("QWENASR_B200_STREAM_K");
        h->stream_k = sk && std::strcmp(sk, "1") == 0;
        const char *rs = getenv("QWENASR_B200_RESIDUAL_SLICES");
        h->res_slices = rs && std::strcmp(rs, "1") == 0;
        const char *aa = getenv("QWENASR_B200_APPEND_AHEAD");
        h->append_ahead = !(aa && std::strcmp(aa, "0") == 0);
    }
    CK(prepare_dense(std::max(c.hidden, std::max(c.intermediate, kQDim))));
    (void)gemm_tc_supported(1, 1, 64);   // resolve the tensor-map encoder before any capture
    CK(cudaStreamSynchronize(h->stream));
    return QKV_OK;
}

void destroy(qkv_handle *h) {
    if (!h) return;
    cudaSetDevice(h->device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    for (auto &L : h->layers) {
        cudaFree(L.attn_norm); cudaFree(L.ffn_norm); cudaFree(L.q_norm); cudaFree(L.k_norm);
        cudaFree(L.w_qkv); cudaFree(L.w_o); cudaFree(L.w_gu); cudaFree(L.w_down);
        cudaFree(L.s_qkv); cudaFree(L.s_o); cudaFree(L.s_gu); cudaFree(L.s_down);
    }
    cudaFree(h->embd); cudaFree(h->w_out); cudaFree(h->out_norm);
    cudaFree(h->ap_norm_w); cudaFree(h->ap_norm_b); cudaFree(h->ap_w0); cudaFree(h->ap_b0); cudaFree(h->ap_w1);
    cudaFree(h->ap_b1);
    cudaFree(h->pool); cudaFree(h->scales); cudaFree(h->d_page_table); cudaFree(h->d_rope);
    cudaFree(h->x); cudaFree(h->qkv); cudaFree(h->res_sl); cudaFree(h->sk_ws); cudaFree(h->sk_flags); cudaFree(h->q); cudaFree(h->q_alt); cudaFree(h->gu); cudaFree(h->logits);
    cudaFree(h->am_v); cudaFree(h->am_i); cudaFree(h->am_cnt);
    cudaFree(h->am_keys); cudaFree(h->am_rcnt); cudaFree(h->d_wout_norm);
    cudaFree(h->xn); cudaFree(h->attn); cudaFree(h->act); cudaFree(h->host_stage); cudaFree(h->qkv_sl);
    cudaFree(h->d_rowbuf); cudaFree(h->d_out_ids); cudaFree(h->d_items); cudaFree(h->part_o); cudaFree(h->part_ml);
    cudaFree(h->counters); cudaFree(h->d_err);
    cudaFreeHost(h->h_page_table); cudaFreeHost(h->h_items); cudaFreeHost(h->h_rowbuf); cudaFreeHost(h->h_out_ids); cudaFreeHost(h->h_err);
    cudaFreeHost(h->h_dec); cudaFree(h->d_dec); cudaFreeHost(h->h_rowptr); cudaFree(h->d_rowptr);
    if (h->dec_ev) cudaEventDestroy(h->dec_ev);
    for (int i = 0; i < qkv_handle::kEmbRing; ++i) {
        cudaFreeHost(h->h_emb[i]);
        if (h->emb_ev[i]) cudaEventDestroy(h->emb_ev[i]);
    }
    for (auto &kv : h->decode_graphs) cudaGraphExecDestroy(kv.second.exec);
    for (auto &kv : h->kv_graphs) cudaGraphExecDestroy(kv.second.exec);
    for (auto &kv : h->kvh_graphs) cudaGraphExecDestroy(kv.second.exec);
    for (auto &ev : h->row_ev) {
        if (ev) cudaEventDestroy(ev);
    }
    if (h->items_ev) cudaEventDestroy(h->items_ev);
    for (cudaEvent_t ev : h->ev_in) cudaEventDestroy(ev);
    for (cudaEvent_t ev : h->ev_done) cudaEventDestroy(ev);
    if (h->ev_tail) cudaEventDestroy(h->ev_tail);
    if (h->copy_in) cudaStreamDestroy(h->copy_in);
    if (h->copy_out) cudaStreamDestroy(h->copy_out);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h->pager;
    delete h;
}

// ---- weights ----

struct Uploader {
    qkv_handle *h;
    void *staging = nullptr;
    size_t staging_bytes = size_t{64} << 20;
    ~Uploader() { cudaFree(staging); }

    // Copy a GGUF tensor (f32/f16/bf16) to dst (+dst_off elements) in dtype.
    int put(const GgufTensor *t, void *dst, int dtype, size_t dst_off) {
        if (t->type == kGgmlI8) return fail(h, QKV_ERR_FORMAT, "tensor holds e4m3 codes; load it with FP8 weights: " + t->name);
        if (!staging) CK(cudaMalloc(&staging, staging_bytes));
        const size_t es = ggml_type_size(t->type);
        const int src_code = t->type == kGgmlF32 ? 0 : t->type == kGgmlF16 ? 1 : 2;
        const size_t n = t->nbytes / es;
        const size_t chunk = staging_bytes / es;
        const size_t out_es = dtype == kActF32 ? 4 : 2;
        for (size_t off = 0; off < n; off += chunk) {
            const size_t cnt = std::min(chunk, n - off);
            CK(cudaMemcpyAsync(staging, t->data + off * es, cnt * es, cudaMemcpyHostToDevice, h->stream));
            CK(launch_convert(staging, src_code, static_cast<uint8_t *>(dst) + (dst_off + off) * out_es, dtype, cnt,
                              h->stream));
            CK(cudaStreamSynchronize(h->stream));   // staging is reused
        }
        return QKV_OK;
    }
};

int find_tensor(qkv_handle *h, const GgufFile &f, const std::string &name, const std::vector<int64_t> &ne,
                const GgufTensor **out) {
    const GgufTensor *t = f.find(name);
    if (!t) return fail(h, QKV_ERR_FORMAT, "missing GGUF tensor: " + name);
    if (ggml_type_size(t->type) == 0) return fail(h, QKV_ERR_FORMAT, "tensor is not f32/f16/bf16: " + name);
    if (t->ne != ne) return fail(h, QKV_ERR_FORMAT, "tensor shape mismatch: " + name);
    *out = t;
    return QKV_OK;
}

// Names and shapes as text-decoder.cpp:191-228 and :523-537 (GGML ne = [in, out]).
int load_weights(qkv_handle *h, const GgufFile &f) {
    const qkv_model_config &c = h->cfg;
    const int64_t H = c.hidden, QD = kQDim, KD = kKvDim, F = c.intermediate, V = c.vocab, D = kHeadDim;
    if (h->proj_fp8 && (H % 128 != 0 || F % 128 != 0 || H > rows_q8_max_k() || F > rows_q8_max_k()))
        return fail(h, QKV_ERR_INVALID_ARG,
                    "FP8 weights need hidden and intermediate sizes that are multiples of 128 and at most 6144");
    // FP8 projection files: every projection an I8 tensor of e4m3 codes with
    // "<name>.scale" (f32, one per row), declared by a metadata key.
    std::string proj_format;
    const bool file_fp8 = f.get_str("qwen3-asr.b200.projections", &proj_format);
    if (file_fp8 && proj_format != "e4m3-row-scale")
        return fail(h, QKV_ERR_FORMAT, "unknown projection format: " + proj_format);
    auto find_codes = [&](const GgufTensor *t, const std::string &name, int64_t rows, const GgufTensor **scale) -> int {
        if (t->type != kGgmlI8) return fail(h, QKV_ERR_FORMAT, "FP8 projection file: not an e4m3 code tensor: " + name);
        const GgufTensor *s = f.find(name + ".scale");
        if (!s || s->type != kGgmlF32 || s->ne != std::vector<int64_t>{rows})
            return fail(h, QKV_ERR_FORMAT, "FP8 projection file: missing or malformed " + name + ".scale");
        *scale = s;
        return QKV_OK;
    };
    const size_t we = h->w_elem;
    Uploader up{h};
    struct DevBuf {
        void *p = nullptr;
        ~DevBuf() { cudaFree(p); }
    } gu_buf;                                   // gate | up as read, before interleaving
    void *&gu_tmp = gu_buf.p;
    h->layers.resize(static_cast<size_t>(c.n_layers));
    int rc;
    for (int l = 0; l < c.n_layers; ++l) {
        const std::string p = "text.blk." + std::to_string(l) + ".";
        const GgufTensor *an, *fn, *wq, *wk, *wv, *wo, *qn, *kn, *wg, *wu, *wd;
        if ((rc = find_tensor(h, f, p + "attn_norm.weight", {H}, &an)) ||
            (rc = find_tensor(h, f, p + "ffn_norm.weight", {H}, &fn)) ||
            (rc = find_tensor(h, f, p + "attn_q.weight", {H, QD}, &wq)) ||
            (rc = find_tensor(h, f, p + "attn_k.weight", {H, KD}, &wk)) ||
            (rc = find_tensor(h, f, p + "attn_v.weight", {H, KD}, &wv)) ||
            (rc = find_tensor(h, f, p + "attn_output.weight", {QD, H}, &wo)) ||
            (rc = find_tensor(h, f, p + "attn_q_norm.weight", {D}, &qn)) ||
            (rc = find_tensor(h, f, p + "attn_k_norm.weight", {D}, &kn)) ||
            (rc = find_tensor(h, f, p + "ffn_gate.weight", {H, F}, &wg)) ||
            (rc = find_tensor(h, f, p + "ffn_up.weight", {H, F}, &wu)) ||
            (rc = find_tensor(h, f, p + "ffn_down.weight", {F, H}, &wd)))
            return rc;
        qkv_handle::Layer &L = h->layers[static_cast<size_t>(l)];
        if (file_fp8) {
            // FP8 projection file: e4m3 codes and row scales go up as stored.
            if (!h->proj_fp8) return fail(h, QKV_ERR_FORMAT, "the file holds FP8 projections: create with FP8 weights");
            const GgufTensor *sq, *sk, *sv, *so, *sg, *su, *sd;
            if ((rc = find_codes(wq, p + "attn_q.weight", QD, &sq)) || (rc = find_codes(wk, p + "attn_k.weight", KD, &sk)) ||
                (rc = find_codes(wv, p + "attn_v.weight", KD, &sv)) ||
                (rc = find_codes(wo, p + "attn_output.weight", H, &so)) ||
                (rc = find_codes(wg, p + "ffn_gate.weight", F, &sg)) ||
                (rc = find_codes(wu, p + "ffn_up.weight", F, &su)) || (rc = find_codes(wd, p + "ffn_down.weight", H, &sd)))
                return rc;
            CK(cudaMalloc(&L.attn_norm, H * sizeof(float)));
            CK(cudaMalloc(&L.ffn_norm, H * sizeof(float)));
            CK(cudaMalloc(&L.q_norm, D * sizeof(float)));
            CK(cudaMalloc(&L.k_norm, D * sizeof(float)));
            CK(cudaMalloc(&L.w_qkv, static_cast<size_t>(QD + 2 * KD) * H));
            CK(cudaMalloc(&L.s_qkv, static_cast<size_t>(QD + 2 * KD) * sizeof(float)));
            CK(cudaMalloc(&L.w_o, static_cast<size_t>(H) * QD));
            CK(cudaMalloc(&L.s_o, static_cast<size_t>(H) * sizeof(float)));
            CK(cudaMalloc(&L.w_gu, static_cast<size_t>(2 * F) * H));
            CK(cudaMalloc(&L.s_gu, static_cast<size_t>(2 * F) * sizeof(float)));
            CK(cudaMalloc(&L.w_down, static_cast<size_t>(H) * F));
            CK(cudaMalloc(&L.s_down, static_cast<size_t>(H) * sizeof(float)));
            if ((rc = up.put(an, L.attn_norm, kActF32, 0)) || (rc = up.put(fn, L.ffn_norm, kActF32, 0)) ||
                (rc = up.put(qn, L.q_norm, kActF32, 0)) || (rc = up.put(kn, L.k_norm, kActF32, 0)))
                return rc;
            auto raw = [&](const GgufTensor *t, void *dst, size_t off) -> int {
                CK(cudaMemcpy(static_cast<uint8_t *>(dst) + off, t->data, t->nbytes, cudaMemcpyHostToDevice));
                return QKV_OK;
            };
            if ((rc = raw(wq, L.w_qkv, 0)) || (rc = raw(wk, L.w_qkv, static_cast<size_t>(QD) * H)) ||
                (rc = raw(wv, L.w_qkv, static_cast<size_t>(QD + KD) * H)) || (rc = raw(sq, L.s_qkv, 0)) ||
                (rc = raw(sk, L.s_qkv, static_cast<size_t>(QD) * 4)) || (rc = raw(sv, L.s_qkv, static_cast<size_t>(QD + KD) * 4)) ||
                (rc = raw(wo, L.w_o, 0)) || (rc = raw(so, L.s_o, 0)) || (rc = raw(wd, L.w_down, 0)) ||
                (rc = raw(sd, L.s_down, 0)))
                return rc;
            // gate | up codes and scales interleaved row by row, as the bf16 layout
            const size_t row = static_cast<size_t>(H);
            CK(cudaMemcpy2D(L.w_gu, 2 * row, wg->data, row, row, static_cast<size_t>(F), cudaMemcpyHostToDevice));
            CK(cudaMemcpy2D(static_cast<uint8_t *>(L.w_gu) + row, 2 * row, wu->data, row, row, static_cast<size_t>(F),
                            cudaMemcpyHostToDevice));
            CK(cudaMemcpy2D(L.s_gu, 2 * sizeof(float), sg->data, sizeof(float), sizeof(float), static_cast<size_t>(F),
                            cudaMemcpyHostToDevice));
            CK(cudaMemcpy2D(L.s_gu + 1, 2 * sizeof(float), su->data, sizeof(float), sizeof(float), static_cast<size_t>(F),
                            cudaMemcpyHostToDevice));
            continue;
        }
        CK(cudaMalloc(&L.attn_norm, H * sizeof(float)));
        CK(cudaMalloc(&L.ffn_norm, H * sizeof(float)));
        CK(cudaMalloc(&L.q_norm, D * sizeof(float)));
        CK(cudaMalloc(&L.k_norm, D * sizeof(float)));
        CK(cudaMalloc(&L.w_qkv, static_cast<size_t>(QD + 2 * KD) * H * we));
        CK(cudaMalloc(&L.w_o, static_cast<size_t>(H) * QD * we));
        CK(cudaMalloc(&L.w_gu, static_cast<size_t>(2 * F) * H * we));
        if (!gu_tmp) CK(cudaMalloc(&gu_tmp, static_cast<size_t>(2 * F) * H * we));
        CK(cudaMalloc(&L.w_down, static_cast<size_t>(H) * F * we));
        if ((rc = up.put(an, L.attn_norm, kActF32, 0)) || (rc = up.put(fn, L.ffn_norm, kActF32, 0)) ||
            (rc = up.put(qn, L.q_norm, kActF32, 0)) || (rc = up.put(kn, L.k_norm, kActF32, 0)) ||
            (rc = up.put(wq, L.w_qkv, h->w_dtype, 0)) ||
            (rc = up.put(wk, L.w_qkv, h->w_dtype, static_cast<size_t>(QD) * H)) ||
            (rc = up.put(wv, L.w_qkv, h->w_dtype, static_cast<size_t>(QD + KD) * H)) ||
            (rc = up.put(wo, L.w_o, h->w_dtype, 0)) || (rc = up.put(wg, gu_tmp, h->w_dtype, 0)) ||
            (rc = up.put(wu, gu_tmp, h->w_dtype, static_cast<size_t>(F) * H)) ||
            (rc = up.put(wd, L.w_down, h->w_dtype, 0)))
            return rc;
        // gate | up -> interleaved row by row: row 2f = gate feature f, row 2f + 1 =
        // up feature f (the layout the fused SwiGLU epilogue of the projection
        // GEMM, the SwiGLU kernel and the e4m3 row quantiser read).
        const size_t row = static_cast<size_t>(H) * we;
        CK(cudaMemcpy2DAsync(L.w_gu, 2 * row, gu_tmp, row, row, static_cast<size_t>(F), cudaMemcpyDeviceToDevice,
                             h->stream));
        CK(cudaMemcpy2DAsync(static_cast<uint8_t *>(L.w_gu) + row, 2 * row,
                             static_cast<const uint8_t *>(gu_tmp) + static_cast<size_t>(F) * H * we, row, row,
                             static_cast<size_t>(F), cudaMemcpyDeviceToDevice, h->stream));
        CK(cudaStreamSynchronize(h->stream));
        if (h->proj_fp8) {
            // FP8 projections: e4m3 codes with one scale per weight row (amax / 448),
            // quantised on the device from the bf16 values just uploaded.
            auto to_fp8 = [&](void *&w, float *&sc, int64_t rows, int64_t K) -> int {
                void *codes = nullptr;
                CK(cudaMalloc(&codes, static_cast<size_t>(rows * K)));
                CK(cudaMalloc(&sc, static_cast<size_t>(rows) * sizeof(float)));
                CK(launch_rows_q8(0, w, static_cast<int>(rows), static_cast<int>(K), nullptr, 0.0f, codes, sc, h->stream));
                CK(cudaStreamSynchronize(h->stream));
                cudaFree(w);
                w = codes;
                return QKV_OK;
            };
            if ((rc = to_fp8(L.w_qkv, L.s_qkv, QD + 2 * KD, H)) || (rc = to_fp8(L.w_o, L.s_o, H, QD)) ||
                (rc = to_fp8(L.w_gu, L.s_gu, 2 * F, H)) || (rc = to_fp8(L.w_down, L.s_down, H, F)))
                return rc;
        }
    }
    const GgufTensor *te, *on, *ow;
    if ((rc = find_tensor(h, f, "text.token_embd.weight", {H, V}, &te)) ||
        (rc = find_tensor(h, f, "text.output_norm.weight", {H}, &on)) ||
        (rc = find_tensor(h, f, "text.output.weight", {H, V}, &ow)))
        return rc;
    CK(cudaMalloc(&h->embd, static_cast<size_t>(V) * H * we));
    CK(cudaMalloc(&h->w_out, static_cast<size_t>(V) * H * we));
    CK(cudaMalloc(&h->out_norm, H * sizeof(float)));
    if ((rc = up.put(te, h->embd, h->w_dtype, 0)) || (rc = up.put(ow, h->w_out, h->w_dtype, 0)) ||
        (rc = up.put(on, h->out_norm, kActF32, 0)))
        return rc;
    if (h->w_dtype == kActBF16) CK(launch_row_norm_max(h->w_out, static_cast<int>(V), static_cast<int>(H), h->d_wout_norm, h->stream));
    // Audio projector, when the file has it (names and shapes of
    // audio-encoder.cpp:776-790; GGML ne = [in, out]).
    if (const GgufTensor *pw0 = f.find("audio.post_norm.weight")) {
        const int64_t A = pw0->ne.size() == 1 ? pw0->ne[0] : 0;
        if (A <= 0 || A % 64 != 0) return fail(h, QKV_ERR_FORMAT, "audio projector width must be a multiple of 64");
        const GgufTensor *pw, *pb, *w0, *b0, *w1, *b1;
        if ((rc = find_tensor(h, f, "audio.post_norm.weight", {A}, &pw)) ||
            (rc = find_tensor(h, f, "audio.post_norm.bias", {A}, &pb)) ||
            (rc = find_tensor(h, f, "audio.proj.0.weight", {A, A}, &w0)) ||
            (rc = find_tensor(h, f, "audio.proj.0.bias", {A}, &b0)) ||
            (rc = find_tensor(h, f, "audio.proj.1.weight", {A, H}, &w1)) ||
            (rc = find_tensor(h, f, "audio.proj.1.bias", {H}, &b1)))
            return rc;
        CK(cudaMalloc(&h->ap_norm_w, A * sizeof(float)));
        CK(cudaMalloc(&h->ap_norm_b, A * sizeof(float)));
        CK(cudaMalloc(&h->ap_w0, static_cast<size_t>(A) * A * we));
        CK(cudaMalloc(&h->ap_b0, A * sizeof(float)));
        CK(cudaMalloc(&h->ap_w1, static_cast<size_t>(H) * A * we));
        CK(cudaMalloc(&h->ap_b1, H * sizeof(float)));
        if ((rc = up.put(pw, h->ap_norm_w, kActF32, 0)) || (rc = up.put(pb, h->ap_norm_b, kActF32, 0)) ||
            (rc = up.put(w0, h->ap_w0, h->w_dtype, 0)) || (rc = up.put(b0, h->ap_b0, kActF32, 0)) ||
            (rc = up.put(w1, h->ap_w1, h->w_dtype, 0)) || (rc = up.put(b1, h->ap_b1, kActF32, 0)))
            return rc;
        h->audio_hidden = static_cast<int>(A);
    }
    h->has_weights = true;
    return QKV_OK;
}

// ---- per-call helpers ----

int check_device_error(qkv_handle *h) {
    CK(cudaMemcpyAsync(h->h_err, h->d_err, sizeof(DevError), cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    if (h->h_err->code != 0) {
        const DevError e = *h->h_err;
        CK(cudaMemsetAsync(h->d_err, 0, sizeof(DevError), h->stream));
        CK(cudaStreamSynchronize(h->stream));
        static const char *what[] = {"", "page index out of range", "bounded wait ran out", "position out of range",
                                     "row out of bounds"};
        const char *w = (e.code >= 0 && e.code <= 4) ? what[e.code] : "unknown";
        return fail(h, QKV_ERR_DEVICE, std::string("device error: ") + w + " (kernel " + std::to_string(e.where) +
                                           ", " + std::to_string(e.a) + ", " + std::to_string(e.b) + ")");
    }
    return QKV_OK;
}

int stream_len(qkv_handle *h, int32_t s) {
    int32_t t = 0;
    h->pager->length(s, &t, nullptr);
    return t;
}

// Prefill attention items: per stream chunk of <= 64 consecutive prompt rows
// (one stream each), per kv head.  Uploaded from pinned staging on the
// handle's stream (prefill calls are synchronous, so the staging is free).
// Row index of stream i's first prompt row in a batch laid out stream by stream.
static int t_first(int i, const int32_t *lens) {
    int t = 0;
    for (int k = 0; k < i; ++k) t += lens[k];
    return t;
}

// Prefill attention work items (first row, queries <= 64, kv head), ordered by
// the number of keys they attend to, longest first: K3's persistent CTAs take
// items round-robin, so this balances them.  base[i] = the stream's position
// of its first query row (nullptr: 0).
int upload_items(qkv_handle *h, int n, const int32_t *lens, const int *base, int *n_items, cudaStream_t st) {
    // h_items is rewritten only after the copy that last read it has run.
    cudaEventSynchronize(h->items_ev);
    // Item order (the persistent K3 CTAs take items round-robin): the items of
    // one (stream, kv head) pair back to back, longest first, pairs of the
    // longest streams first.  A pair's query blocks then run at the same time
    // on neighbouring CTAs and share its K/V tiles through L2, and each CTA
    // still sees every block length in turn.  QWENASR_B200_K3_ORDER=lpt keeps
    // the plain longest-first order over all items (the earlier schedule).
    static const bool lpt = [] {
        const char *e = std::getenv("QWENASR_B200_K3_ORDER");
        return e && std::strcmp(e, "lpt") == 0;
    }();
    struct Tagged {
        int total, stream, g;
        int4 it;
    };
    std::vector<Tagged> v;
    int row = 0;
    for (int i = 0; i < n; ++i) {
        const int total = (base ? base[i] : 0) + lens[i];
        for (int q0 = 0; q0 < lens[i]; q0 += 64) {
            const int nq = std::min(64, lens[i] - q0);
            const int keys = (base ? base[i] : 0) + q0 + nq;
            for (int g = 0; g < kHkv; ++g) {
                if (static_cast<int>(v.size()) >= h->max_items)
                    return fail(h, QKV_ERR_CAPACITY, "too many prefill attention items");
                v.push_back({total, i, g, make_int4(row + q0, nq, g, keys)});
            }
        }
        row += lens[i];
    }
    if (lpt) {
        std::stable_sort(v.begin(), v.end(), [](const Tagged &a, const Tagged &b) { return a.it.w > b.it.w; });
    } else {
        std::stable_sort(v.begin(), v.end(), [](const Tagged &a, const Tagged &b) {
            if (a.total != b.total) return a.total > b.total;
            if (a.stream != b.stream) return a.stream < b.stream;
            if (a.g != b.g) return a.g < b.g;
            return a.it.w > b.it.w;
        });
    }
    const int k = static_cast<int>(v.size());
    for (int j = 0; j < k; ++j) h->h_items[j] = v[static_cast<size_t>(j)].it;
    CK(cudaMemcpyAsync(h->d_items, h->h_items, static_cast<size_t>(k) * sizeof(int4), cudaMemcpyHostToDevice, st));
    CK(cudaEventRecord(h->items_ev, st));
    *n_items = k;
    return QKV_OK;
}

// Grow each row's stream by `tokens` (pages from the pager) and push changed
// page-table rows to the device.
int grow_streams(qkv_handle *h, int n, const int32_t *streams, const int32_t *tokens, cudaStream_t st) {
    // All-or-nothing for the batch: check the page budget first.
    int64_t need = 0;
    for (int i = 0; i < n; ++i) {
        const int64_t len = stream_len(h, streams[i]);
        const int64_t t = tokens ? tokens[i] : 1;
        const int64_t have = static_cast<int64_t>(h->pager->pages(streams[i])->size());
        const int64_t want = (len + t + kPageTokens - 1) / kPageTokens;
        if (want > h->maxp) return fail(h, QKV_ERR_CAPACITY, "stream would exceed max_context pages");
        need += want - have;
    }
    if (need > h->pager->free_pages()) {
        return fail(h, QKV_ERR_OUT_OF_PAGES, "KV pool out of pages (need " + std::to_string(need) + ", free " +
                                                 std::to_string(h->pager->free_pages()) + ")");
    }
    std::vector<int32_t> added;
    for (int i = 0; i < n; ++i) {
        added.clear();
        std::string e;
        const int rc = h->pager->append(streams[i], tokens ? tokens[i] : 1, &added, &e);
        if (rc != QKV_OK) return fail(h, rc, e);
        if (!added.empty()) {
            const std::vector<int32_t> *pg = h->pager->pages(streams[i]);
            const size_t first = pg->size() - added.size();
            int *row = h->h_page_table + static_cast<size_t>(streams[i]) * h->maxp;
            for (size_t k = first; k < pg->size(); ++k) row[k] = (*pg)[k];
            CK(cudaMemcpyAsync(h->d_page_table + static_cast<size_t>(streams[i]) * h->maxp + first, row + first,
                               added.size() * sizeof(int), cudaMemcpyHostToDevice, st));
        }
    }
    return QKV_OK;
}

// Pinned staging for the per-call row arrays.  A slot is reused only after the
// copy that last read it has run (its event), so callers never block on the
// previous step's kernels.
int *row_stage(qkv_handle *h) {
    h->row_slot = (h->row_slot + 1) % qkv_handle::kRowRing;
    cudaEventSynchronize(h->row_ev[h->row_slot]);
    return h->h_rowbuf + static_cast<size_t>(h->row_slot) * 4 * h->max_rows;
}

int row_upload(qkv_handle *h, const int *host, size_t count, cudaStream_t st) {
    CK(cudaMemcpyAsync(h->d_rowbuf, host, count * sizeof(int), cudaMemcpyHostToDevice, st));
    CK(cudaEventRecord(h->row_ev[h->row_slot], st));
    return QKV_OK;
}

// Prompt rows (stream i: rows[i], lens[i] rows of `row_floats` f32, host
// memory) -> dst (device, rows back to back) through the pinned chunk ring.
// Each chunk is filled by up to kFillThreads threads (byte ranges of equal
// size, across row-block boundaries) and sent with one asynchronous copy, so
// the fill of one chunk overlaps the copy of the other.
int upload_prompt_rows(qkv_handle *h, float *dst, int n, const float *const *rows, const int32_t *lens,
                       int row_floats, cudaStream_t st) {
    constexpr int kFillThreads = 8;
    constexpr size_t kBytesPerThread = size_t(1) << 20;
    const size_t row_bytes = static_cast<size_t>(row_floats) * sizeof(float);
    if (row_bytes == 0 || row_bytes > qkv_handle::kEmbChunkBytes || !h->h_emb[0])
        return fail(h, QKV_ERR_STATE, "prompt staging: no pinned chunks or rows wider than a chunk");
    struct Seg {
        const uint8_t *src;
        size_t bytes, off;   // off: byte offset inside the chunk
    };
    std::vector<Seg> segs;
    size_t dst_off = 0;   // bytes of dst written so far
    int i = 0;
    size_t in_row = 0;    // bytes of stream i already taken
    while (i < n) {
        // gather up to one chunk of whole rows (at least one row)
        segs.clear();
        size_t fill = 0;
        while (i < n) {
            const size_t total_i = static_cast<size_t>(lens[i]) * row_bytes;
            const size_t room = (qkv_handle::kEmbChunkBytes - fill) / row_bytes * row_bytes;
            if (room == 0) break;
            const size_t take = std::min(total_i - in_row, room);
            if (take > 0) segs.push_back({reinterpret_cast<const uint8_t *>(rows[i]) + in_row, take, fill});
            fill += take;
            in_row += take;
            if (in_row == total_i) {
                ++i;
                in_row = 0;
            }
        }
        if (fill == 0) break;
        const int slot = h->emb_slot;
        h->emb_slot = (slot + 1) % qkv_handle::kEmbRing;
        CK(cudaEventSynchronize(h->emb_ev[slot]));
        uint8_t *chunk = reinterpret_cast<uint8_t *>(h->h_emb[slot]);
        auto copy_range = [&](size_t lo, size_t hi) {   // chunk bytes [lo, hi)
            for (const Seg &g : segs) {
                const size_t a = std::max(lo, g.off), b = std::min(hi, g.off + g.bytes);
                if (a < b) std::memcpy(chunk + a, g.src + (a - g.off), b - a);
            }
        };
        const int nt = static_cast<int>(std::min<size_t>(kFillThreads, std::max<size_t>(1, fill / kBytesPerThread)));
        if (nt == 1) {
            copy_range(0, fill);
        } else {
            std::vector<std::thread> pool;
            const size_t per = (fill + nt - 1) / nt;
            for (int t = 1; t < nt; ++t)
                pool.emplace_back(copy_range, std::min(fill, per * t), std::min(fill, per * (t + 1)));
            copy_range(0, std::min(fill, per));
            for (auto &th : pool) th.join();
        }
        CK(cudaMemcpyAsync(reinterpret_cast<uint8_t *>(dst) + dst_off, chunk, fill, cudaMemcpyHostToDevice, st));
        CK(cudaEventRecord(h->emb_ev[slot], st));
        dst_off += fill;
    }
    return QKV_OK;
}

// Record `body` (kernel launches on h->stream) into a graph and instantiate it.
int capture_graph(qkv_handle *h, const std::function<int()> &body, qkv_handle::Graph *out) {
    const int64_t launches_before = h->launches;
    CK(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
    const int rc = body();
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(h->stream, &g);
    h->launches = launches_before;
    if (rc != QKV_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(h, e, "cudaStreamEndCapture");
    size_t n_nodes = 0;
    cudaGraphGetNodes(g, nullptr, &n_nodes);
    std::vector<cudaGraphNode_t> nodes(n_nodes);
    cudaGraphGetNodes(g, nodes.data(), &n_nodes);
    int64_t kernels = 0;
    for (cudaGraphNode_t nd : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ei = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    if (ei != cudaSuccess) return cuda_fail(h, ei, "cudaGraphInstantiate");
    out->exec = exec;
    out->kernels = kernels;
    return QKV_OK;
}

int check_streams(qkv_handle *h, int n, const int32_t *streams) {
    if (n <= 0 || !streams) return fail(h, QKV_ERR_INVALID_ARG, "empty batch");
    if (n > h->rt.max_streams) return fail(h, QKV_ERR_CAPACITY, "batch larger than max_streams");
    std::vector<uint8_t> seen(static_cast<size_t>(h->rt.max_streams), 0);
    for (int i = 0; i < n; ++i) {
        if (!h->pager->is_open(streams[i])) return fail(h, QKV_ERR_INVALID_ARG, "stream " + std::to_string(streams[i]) + " is not open");
        if (seen[static_cast<size_t>(streams[i])]++) return fail(h, QKV_ERR_INVALID_ARG, "stream listed twice in one batch");
    }
    return QKV_OK;
}

// Softmax scale folded into q: 1 / sqrt(head dim) in the log2 domain.
float attn_scale_log2() { return static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(kHeadDim))); }

AppendParams append_params(qkv_handle *h, int layer, int n, const int *slots, const int *pos, const float *qkv,
                           float *q_out, const float *qn, const float *kn) {
    AppendParams p{};
    p.n = n;
    p.slots = slots;
    p.positions = pos;
    p.qkv = qkv;
    p.q_out = q_out;
    p.q_norm_w = qn;
    p.k_norm_w = kn;
    p.rope = h->d_rope;
    p.rope_len = h->rope_len;
    p.pool = static_cast<uint8_t *>(h->pool) + h->pool_layer_bytes * static_cast<size_t>(layer);
    p.scales = h->scales ? h->scales + h->scales_layer_elems * static_cast<size_t>(layer) : nullptr;
    p.page_table = h->d_page_table;
    p.maxp = h->maxp;
    p.max_streams = h->rt.max_streams;
    p.n_pages = h->n_pages;
    p.eps = h->cfg.rms_norm_eps;
    p.err = h->d_err;
    p.v_int8 = h->rt.kv_dtype == kKvE4I8 ? 1 : 0;
    p.qkv_slices = 1;
    if (qkv && qkv == h->qkv_sl) {   // the projection left partial-sum slices
        p.qkv_slices = h->qkv_nsl;
        p.qkv_slice_stride = h->qkv_sl_stride;
    }
    return p;
}

AttendParams attend_params(qkv_handle *h, int layer, int n, const int *slots, const int *lens, const float *q,
                           void *out) {
    AttendParams p{};
    p.n = n;
    p.slots = slots;
    p.lens = lens;
    p.q = q;
    p.out = out;
    p.pool = static_cast<uint8_t *>(h->pool) + h->pool_layer_bytes * static_cast<size_t>(layer);
    p.scales = h->scales ? h->scales + h->scales_layer_elems * static_cast<size_t>(layer) : nullptr;
    p.page_table = h->d_page_table;
    p.maxp = h->maxp;
    p.max_streams = h->rt.max_streams;
    p.n_pages = h->n_pages;
    p.part_o = h->part_o;
    p.part_ml = h->part_ml;
    p.counters = h->counters;
    p.scale_log2 = attn_scale_log2();
    p.err = h->d_err;
    return p;
}

// Append + attend for `n` decode rows of one layer (rows: slots/pos/lens device arrays).
int layer_kv(qkv_handle *h, int layer, int n, const int *slots, const int *pos, const int *lens, const float *qkv,
             float *q, void *out, bool out_bf16, const float *qn, const float *kn, cudaStream_t st) {
    AppendParams ap = append_params(h, layer, n, slots, pos, qkv, q, qn, kn);
    CK(launch_kv_append(ap, h->rt.kv_dtype, st));
    AttendParams at = attend_params(h, layer, n, slots, lens, q, out);
    at.early = 1;   // K1 just appended one token per row (see AttendParams::early)
    CK(launch_decode_attn(at, h->rt.kv_dtype, out_bf16, h->num_sms, st));
    h->launches += 2;
    return QKV_OK;
}

// One layer of a KV step whose every layer's projections are on the device
// (qkv_l: this layer's rows; qkv_next: layer l + 1's, or null for the last
// layer).  With the append-ahead, layers 0 .. ahead_from get K1 and the K2 of
// every layer from ahead_from on also appends layer l + 1 (ahead_from 1 lets
// layer 0's attention start on layer 0's inputs alone, for callers whose
// inputs are still arriving); q alternates between two buffers by layer parity.
int kv_step_layer(qkv_handle *h, int l, int n, const int *slots, const int *pos, const int *lens, const float *qkv_l,
                  const float *qkv_next, float *out, cudaStream_t st, int ahead_from = 0) {
    const qkv_handle::Layer &L = h->layers[static_cast<size_t>(l)];
    if (!h->append_ahead) return layer_kv(h, l, n, slots, pos, lens, qkv_l, h->q, out, false, L.q_norm, L.k_norm, st);
    float *q_cur = (l & 1) ? h->q_alt : h->q;
    float *q_next = (l & 1) ? h->q : h->q_alt;
    if (l <= ahead_from) {
        CK(launch_kv_append(append_params(h, l, n, slots, pos, qkv_l, q_cur, L.q_norm, L.k_norm), h->rt.kv_dtype, st));
        h->launches += 1;
    }
    AttendParams at = attend_params(h, l, n, slots, lens, q_cur, out);
    at.early = 1;   // the kernel before (K1 or K2 of layer l - 1) wrote only each row's last page of this layer
    if (qkv_next && l >= ahead_from) {
        const qkv_handle::Layer &Ln = h->layers[static_cast<size_t>(l + 1)];
        at.next = append_params(h, l + 1, n, slots, pos, qkv_next, q_next, Ln.q_norm, Ln.k_norm);
    }
    CK(launch_decode_attn(at, h->rt.kv_dtype, false, h->num_sms, st));
    h->launches += 1;
    return QKV_OK;
}

// Projection C (+)= X . W^T: tcgen05 when activations and weights are bf16,
// the SIMT kernel otherwise (f32 parity mode).
cudaError_t gemm(qkv_handle *h, const void *X, const void *W, float *C, int M, int N, int K, int accumulate) {
    if (h->act_dtype == kActBF16 && h->w_dtype == kActBF16 && gemm_tc_supported(M, N, K)) {
        h->launches += gemm_tc_kernels(M, N, K, accumulate, h->num_sms) - 1;   // the zeroing kernel, if any
        return launch_gemm_tc(X, W, C, M, N, K, accumulate, h->num_sms, h->d_err, h->stream);
    }
    return launch_gemm(X, h->act_dtype, W, h->w_dtype, C, M, N, K, accumulate, h->stream);
}

// Logits of the rows listed in d_rows (indices into x) -> ids (device), logits into h->logits.
int head_and_argmax(qkv_handle *h, int n, const int *d_rows) {
    const qkv_model_config &c = h->cfg;
    // The final norm also folds the last layer's pending down-projection slices
    // into the rows it reads (x of the other rows is not read again).
    CK(launch_rmsnorm(h->x, d_rows, n, c.hidden, h->out_norm, c.rms_norm_eps, h->xn, h->act_dtype, h->stream,
                      h->res_pending));
    h->res_pending = ResidualFold{};
    CK(gemm(h, h->xn, h->w_out, h->logits, n, c.vocab, c.hidden, 0));
    CK(launch_argmax_split(h->logits, n, c.vocab, h->d_out_ids, h->am_v, h->am_i, h->am_cnt,
                           qkv_handle::kArgmaxSlices, h->num_sms, h->stream));
    h->launches += 3;
    if (h->w_dtype == kActBF16 && h->exact_argmax) {
        // The bf16 head rounds the final hidden row to bf16 (2^-8 relative):
        // re-score, in f32, every token that could be the f32 argmax.
        CK(launch_argmax_refine(h->logits, n, c.vocab, h->x, d_rows, c.hidden, h->out_norm, c.rms_norm_eps, h->w_out,
                                h->d_wout_norm, h->am_keys, h->am_rcnt, h->d_out_ids, h->num_sms, h->stream));
        h->launches += 1;
    }
    return QKV_OK;
}

// All layers over `n` rows whose inputs are in h->x; decode rows attend with
// K2, prompt rows with the causal prefill kernel.
// K3 (tensor cores) serves bf16 and e4m3 caches when items are given.
bool prefill_on_tc(const qkv_handle *h, const int4 *items, int n_items) {
    return h->prefill_tc && prefill_tc_supported(h->rt.kv_dtype) && items && n_items > 0;
}

// Causal prefill attention over layer l's cache for n query rows (slots,
// positions on the device): K3 on the tensor cores for bf16/e4m3 caches
// (items = 64-query blocks per kv head), the CUDA-core kernel otherwise.
// K3 reads q16 (q x scale in its operand type, as K1 writes it for prompt
// rows); when q16 is null, q is converted into it first, into h->q's storage
// behind q (q itself must then not be h->q).
cudaError_t prefill_attend(qkv_handle *h, int l, int n, const int *slots, const int *pos, const float *q,
                           const void *q16, void *out, bool out_bf16, const int4 *items, int n_items, cudaStream_t st) {
    PrefillAttnParams pp{};
    pp.n = n;
    pp.slots = slots;
    pp.positions = pos;
    pp.q = q;
    pp.q16 = q16;
    pp.out = out;
    pp.pool = static_cast<const uint8_t *>(h->pool) + h->pool_layer_bytes * static_cast<size_t>(l);
    pp.scales = h->scales ? h->scales + h->scales_layer_elems * static_cast<size_t>(l) : nullptr;
    pp.page_table = h->d_page_table;
    pp.maxp = h->maxp;
    pp.max_streams = h->rt.max_streams;
    pp.n_pages = h->n_pages;
    pp.scale_log2 = attn_scale_log2();
    pp.err = h->d_err;
    if (prefill_on_tc(h, items, n_items)) {
        if (!pp.q16) {
            cudaError_t e = launch_q_to16(q, n, pp.scale_log2, kv_is_8bit(h->rt.kv_dtype), h->q, st);
            if (e != cudaSuccess) return e;
            pp.q16 = h->q;
        }
        return launch_prefill_attn_tc(pp, h->rt.kv_dtype, items, n_items, out_bf16, st);
    }
    return launch_prefill_attn(pp, h->rt.kv_dtype, out_bf16, st);
}

// FP8 projection: C (+)= (xq x xq_s) . (W x w_s)^T.
cudaError_t gemm8(qkv_handle *h, const void *W, const float *w_s, float *C, int M, int N, int K, int accumulate) {
    h->launches += gemm_tc_fp8_kernels(M, N, K, accumulate, h->num_sms);
    return launch_gemm_tc_fp8(h->xq, h->xq_s, W, w_s, C, M, N, K, accumulate, h->num_sms, h->d_err, h->stream);
}

// The qkv projection of one layer: in slice mode for a decode-sized batch on
// the tensor cores (returns h->qkv_sl), else into h->qkv.
const float *qkv_projection(qkv_handle *h, const qkv_handle::Layer &L, int n, cudaError_t *e) {
    const qkv_model_config &c = h->cfg;
    const bool tc = h->proj_fp8 ? gemm_tc_fp8_supported(n, kQkvDim, c.hidden)
                                : (h->act_dtype == kActBF16 && h->w_dtype == kActBF16 &&
                                   gemm_tc_supported(n, kQkvDim, c.hidden));
    if (tc && h->qkv_sl && n <= h->rt.max_streams) {
        h->qkv_sl_stride = static_cast<size_t>(n) * kQkvDim;
        h->launches += 1;
        *e = h->proj_fp8 ? launch_gemm_tc_fp8_slices(h->xq, h->xq_s, L.w_qkv, L.s_qkv, h->qkv_sl, n, kQkvDim, c.hidden,
                                                     qkv_handle::kQkvMaxSlices, h->num_sms, h->d_err, h->stream,
                                                     &h->qkv_nsl)
                         : launch_gemm_tc_slices(h->xn, L.w_qkv, h->qkv_sl, n, kQkvDim, c.hidden,
                                                 qkv_handle::kQkvMaxSlices, h->num_sms, h->d_err, h->stream, &h->qkv_nsl);
        return h->qkv_sl;
    }
    *e = h->proj_fp8 ? gemm8(h, L.w_qkv, L.s_qkv, h->qkv, n, kQkvDim, c.hidden, 0)
                     : gemm(h, h->xn, L.w_qkv, h->qkv, n, kQkvDim, c.hidden, 0);
    return h->qkv;
}

// The o or down projection of one layer, whose result adds to the residual
// x (X: the bf16 attention output or activation; the FP8 path takes the e4m3
// rows already in xq).  A decode-sized batch on the tensor cores runs in
// slice mode: each K split stores its partial sums into res_sl (plain stores,
// no atomics, x not touched) and the returned fold is added to x, in slice
// order, by the kernel that reads x next.  Otherwise x += X . W^T here and
// the fold is empty.
int residual_projection(qkv_handle *h, const void *W, const float *w_s, const void *X, int n, int K, ResidualFold *fold) {
    const int H = h->cfg.hidden;
    *fold = ResidualFold{};
    const bool tc = h->proj_fp8 ? gemm_tc_fp8_supported(n, H, K)
                                : (h->act_dtype == kActBF16 && h->w_dtype == kActBF16 && gemm_tc_supported(n, H, K));
    if (tc && h->res_slices && h->res_sl && n <= h->rt.max_streams) {
        int nsl = 1;
        CK(h->proj_fp8 ? launch_gemm_tc_fp8_slices(h->xq, h->xq_s, W, w_s, h->res_sl, n, H, K, qkv_handle::kResMaxSlices,
                                                   h->num_sms, h->d_err, h->stream, &nsl)
                       : launch_gemm_tc_slices(X, W, h->res_sl, n, H, K, qkv_handle::kResMaxSlices, h->num_sms, h->d_err,
                                               h->stream, &nsl));
        if (h->proj_fp8) h->launches += 1;   // (the bf16 loop counts its projections itself)
        fold->slices = h->res_sl;
        fold->n = nsl;
        fold->stride = static_cast<size_t>(n) * H;
        return QKV_OK;
    }
    CK(h->proj_fp8 ? gemm8(h, W, w_s, h->x, n, H, K, 1) : gemm(h, X, W, h->x, n, H, K, 1));
    return QKV_OK;
}

// One layer with FP8 projections: every projection input is quantised to
// e4m3 rows with a scale per row by the kernel that builds it (RMSNorm,
// SwiGLU) or right after (the attention output).  fold: in, the residual's
// pending slices (the previous layer's down projection); out, this layer's.
int run_layer_fp8(qkv_handle *h, const qkv_handle::Layer &L, int l, int n, const int *slots, const int *pos,
                  const int *lens, bool prompt, const int4 *items, int n_items, ResidualFold *fold) {
    const qkv_model_config &c = h->cfg;
    const float eps = c.rms_norm_eps;
    int rc;
    CK(launch_rows_q8(1, h->x, n, c.hidden, L.attn_norm, eps, h->xq, h->xq_s, h->stream, *fold));
    cudaError_t pe = cudaSuccess;
    const float *qkv = qkv_projection(h, L, n, &pe);
    CK(pe);
    if (!prompt) {
        if ((rc = layer_kv(h, l, n, slots, pos, lens, qkv, h->q, h->attn, true, L.q_norm, L.k_norm, h->stream)))
            return rc;
    } else {
        const bool tc = prefill_on_tc(h, items, n_items);
        AppendParams ap = append_params(h, l, n, slots, pos, qkv, tc ? nullptr : h->q, L.q_norm, L.k_norm);
        if (tc) {
            ap.q16_out = h->q;
            ap.q16_scale = attn_scale_log2();
            ap.q16_f16 = kv_is_8bit(h->rt.kv_dtype) ? 1 : 0;
        }
        CK(launch_kv_append(ap, h->rt.kv_dtype, h->stream));
        CK(prefill_attend(h, l, n, slots, pos, h->q, tc ? h->q : nullptr, h->attn, true, items, n_items, h->stream));
        h->launches += 2;
    }
    CK(launch_rows_q8(0, h->attn, n, kQDim, nullptr, 0.0f, h->xq, h->xq_s, h->stream));
    if ((rc = residual_projection(h, L.w_o, L.s_o, nullptr, n, kQDim, fold))) return rc;
    CK(launch_rows_q8(1, h->x, n, c.hidden, L.ffn_norm, eps, h->xq, h->xq_s, h->stream, *fold));
    CK(gemm8(h, L.w_gu, L.s_gu, h->gu, n, 2 * c.intermediate, c.hidden, 0));
    CK(launch_rows_q8(2, h->gu, n, c.intermediate, nullptr, 0.0f, h->xq, h->xq_s, h->stream));
    if ((rc = residual_projection(h, L.w_down, L.s_down, nullptr, n, c.intermediate, fold))) return rc;
    h->launches += 4;
    return QKV_OK;
}

int run_layers(qkv_handle *h, int n, const int *slots, const int *pos, const int *lens, bool prompt, int l0 = 0,
               int l1 = -1, const int4 *items = nullptr, int n_items = 0) {
    const qkv_model_config &c = h->cfg;
    const bool bf = h->act_dtype == kActBF16;
    int rc;
    if (l1 < 0) l1 = c.n_layers;
    ResidualFold fold{};   // x is complete on entry (embeddings, decoder input or the caller's rows)
    h->res_pending = ResidualFold{};
    for (int l = l0; l < l1; ++l) {
        const qkv_handle::Layer &L = h->layers[static_cast<size_t>(l)];
        if (h->proj_fp8) {
            if ((rc = run_layer_fp8(h, L, l, n, slots, pos, lens, prompt, items, n_items, &fold))) return rc;
            continue;
        }
        CK(launch_rmsnorm(h->x, nullptr, n, c.hidden, L.attn_norm, c.rms_norm_eps, h->xn, h->act_dtype, h->stream,
                          fold));
        cudaError_t pe = cudaSuccess;
        const float *qkv = qkv_projection(h, L, n, &pe);
        CK(pe);
        if (!prompt) {
            if ((rc = layer_kv(h, l, n, slots, pos, lens, qkv, h->q, h->attn, bf, L.q_norm, L.k_norm, h->stream)))
                return rc;
        } else {
            // K3 takes q from K1 already scaled and rounded to its operand type.
            const bool tc = prefill_on_tc(h, items, n_items);
            AppendParams ap = append_params(h, l, n, slots, pos, qkv, tc ? nullptr : h->q, L.q_norm, L.k_norm);
            if (tc) {
                ap.q16_out = h->q;
                ap.q16_scale = attn_scale_log2();
                ap.q16_f16 = kv_is_8bit(h->rt.kv_dtype) ? 1 : 0;
            }
            CK(launch_kv_append(ap, h->rt.kv_dtype, h->stream));
            CK(prefill_attend(h, l, n, slots, pos, h->q, tc ? h->q : nullptr, h->attn, bf, items, n_items, h->stream));
            h->launches += 2;
        }
        if ((rc = residual_projection(h, L.w_o, nullptr, h->attn, n, kQDim, &fold))) return rc;
        CK(launch_rmsnorm(h->x, nullptr, n, c.hidden, L.ffn_norm, c.rms_norm_eps, h->xn, h->act_dtype, h->stream,
                          fold));
        const bool fused = h->fused_swiglu && h->act_dtype == kActBF16 && h->w_dtype == kActBF16 &&
                           gemm_tc_supported(n, 2 * c.intermediate, c.hidden) &&
                           gemm_tc_swiglu_pays(n, 2 * c.intermediate, c.hidden, h->num_sms);
        if (fused) {
            // gate/up projection with SwiGLU in its epilogue: act (bf16) straight from TMEM
            CK(launch_gemm_tc_swiglu(h->xn, L.w_gu, h->act, n, 2 * c.intermediate, c.hidden, h->num_sms, h->d_err,
                                     h->stream, h->stream_k ? h->sk_ws : nullptr, h->sk_flags, h->sk_ws_floats,
                                     h->sk_flag_tiles));
        } else {
            CK(gemm(h, h->xn, L.w_gu, h->gu, n, 2 * c.intermediate, c.hidden, 0));
            CK(launch_swiglu(h->gu, n, c.intermediate, h->act, h->act_dtype, h->stream));
        }
        if ((rc = residual_projection(h, L.w_down, nullptr, h->act, n, c.intermediate, &fold))) return rc;
        h->launches += fused ? 6 : 7;
    }
    h->res_pending = fold;   // the last down projection: folded by the head (or by the caller)
    return QKV_OK;
}

int finish_ids(qkv_handle *h, int n, const int32_t *streams, int32_t *out_ids, float *out_logits) {
    CK(cudaMemcpyAsync(h->h_out_ids, h->d_out_ids, static_cast<size_t>(n) * sizeof(int), cudaMemcpyDeviceToHost,
                       h->stream));
    if (out_logits) {
        CK(cudaMemcpyAsync(out_logits, h->logits, static_cast<size_t>(n) * h->cfg.vocab * sizeof(float),
                           cudaMemcpyDeviceToHost, h->stream));
    }
    int rc = check_device_error(h);
    if (rc) return rc;
    for (int i = 0; i < n; ++i) {
        const int id = h->h_out_ids[i];
        if (id < 0 || id >= h->cfg.vocab) return fail(h, QKV_ERR_DEVICE, "generated token id is out of range");
        h->last_id[static_cast<size_t>(streams[i])] = id;
        if (out_ids) out_ids[i] = id;
    }
    return QKV_OK;
}

}  // namespace

// =====================================================================
extern "C" {

int qkv_read_gguf_config(const char *gguf_path, qkv_model_config *cfg, char *err, size_t err_len) {
    if (!cfg) {
        set_err(err, err_len, "cfg is null");
        return QKV_ERR_INVALID_ARG;
    }
    GgufFile f;
    std::string e;
    int rc = f.open(gguf_path, &e);
    if (rc) {
        set_err(err, err_len, e);
        return rc;
    }
    uint32_t L, H, Hq, Hkv, D, F, V;
    float theta, eps;
    const bool ok = f.get_u32("qwen3-asr.text.num_hidden_layers", &L) && f.get_u32("qwen3-asr.text.hidden_size", &H) &&
                    f.get_u32("qwen3-asr.text.num_attention_heads", &Hq) &&
                    f.get_u32("qwen3-asr.text.num_key_value_heads", &Hkv) && f.get_u32("qwen3-asr.text.head_dim", &D) &&
                    f.get_u32("qwen3-asr.text.intermediate_size", &F) && f.get_u32("qwen3-asr.text.vocab_size", &V) &&
                    f.get_f32("qwen3-asr.text.rope_theta", &theta) && f.get_f32("qwen3-asr.text.rms_norm_eps", &eps);
    if (!ok) {
        set_err(err, err_len, "GGUF lacks a qwen3-asr.text.* key (or it has the wrong type)");
        return QKV_ERR_FORMAT;
    }
    cfg->n_layers = static_cast<int32_t>(L);
    cfg->hidden = static_cast<int32_t>(H);
    cfg->n_heads = static_cast<int32_t>(Hq);
    cfg->n_kv_heads = static_cast<int32_t>(Hkv);
    cfg->head_dim = static_cast<int32_t>(D);
    cfg->intermediate = static_cast<int32_t>(F);
    cfg->vocab = static_cast<int32_t>(V);
    cfg->rope_theta = theta;
    cfg->rms_norm_eps = eps;
    return QKV_OK;
}

int qkv_create(const char *gguf_path, const qkv_model_config *cfg, const qkv_runtime_config *rt, qkv_handle **out,
               char *err, size_t err_len) {
    const TraceRange trace("qkv_create");
    if (!out || !rt) {
        set_err(err, err_len, "out or rt is null");
        return QKV_ERR_INVALID_ARG;
    }
    *out = nullptr;
    qkv_model_config c{};
    int rc;
    if (cfg) {
        c = *cfg;
    } else if ((rc = qkv_read_gguf_config(gguf_path, &c, err, err_len)) != QKV_OK) {
        return rc;
    }
    std::string e;
    if ((rc = validate_model(c, &e)) || (rc = validate_rt(*rt, &e))) {
        set_err(err, err_len, e);
        return rc;
    }
    GgufFile f;
    if ((rc = f.open(gguf_path, &e))) {
        set_err(err, err_len, e);
        return rc;
    }
    qkv_handle *h = new qkv_handle();
    h->cfg = c;
    h->rt = *rt;
    h->proj_fp8 = rt->weight_dtype == QKV_FP8_E4M3;
    h->w_dtype = rt->weight_dtype == QKV_F32 ? kActF32 : kActBF16;
    h->act_dtype = h->w_dtype;
    h->w_elem = h->w_dtype == kActBF16 ? 2 : 4;
    if ((rc = host_alloc_guard(h, [&] { return setup_common(h, true); })) ||
        (rc = host_alloc_guard(h, [&] { return load_weights(h, f); }))) {
        set_err(err, err_len, h->last_error);
        destroy(h);
        return rc;
    }
    *out = h;
    return QKV_OK;
}

int qkv_create_kv_only(const qkv_model_config *cfg, const qkv_runtime_config *rt, const float *q_norm_w,
                       const float *k_norm_w, qkv_handle **out, char *err, size_t err_len) {
    if (!out || !rt || !cfg || !q_norm_w || !k_norm_w) {
        set_err(err, err_len, "null argument");
        return QKV_ERR_INVALID_ARG;
    }
    *out = nullptr;
    std::string e;
    int rc;
    if ((rc = validate_model(*cfg, &e)) || (rc = validate_rt(*rt, &e))) {
        set_err(err, err_len, e);
        return rc;
    }
    qkv_handle *h = new qkv_handle();
    h->cfg = *cfg;
    h->rt = *rt;
    h->w_dtype = kActF32;
    h->act_dtype = kActF32;
    if ((rc = host_alloc_guard(h, [&] { return setup_common(h, false); }))) {
        set_err(err, err_len, h->last_error);
        destroy(h);
        return rc;
    }
    h->layers.resize(static_cast<size_t>(cfg->n_layers));
    for (int l = 0; l < cfg->n_layers; ++l) {
        qkv_handle::Layer &L = h->layers[static_cast<size_t>(l)];
        if (cudaMalloc(&L.q_norm, kHeadDim * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&L.k_norm, kHeadDim * sizeof(float)) != cudaSuccess ||
            cudaMemcpy(L.q_norm, q_norm_w + static_cast<size_t>(l) * kHeadDim, kHeadDim * sizeof(float),
                       cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(L.k_norm, k_norm_w + static_cast<size_t>(l) * kHeadDim, kHeadDim * sizeof(float),
                       cudaMemcpyHostToDevice) != cudaSuccess) {
            set_err(err, err_len, "failed to upload QK-norm weights");
            destroy(h);
            return QKV_ERR_CUDA;
        }
    }
    *out = h;
    return QKV_OK;
}

void qkv_destroy(qkv_handle *h) { destroy(h); }

const char *qkv_last_error(const qkv_handle *h) { return h ? h->last_error.c_str() : "null handle"; }

int qkv_stream_open(qkv_handle *h, int32_t *stream_id) {
    if (!h) return QKV_ERR_INVALID_ARG;
    std::string e;
    const int rc = h->pager->open(stream_id, &e);
    if (rc) return fail(h, rc, e);
    h->last_id[static_cast<size_t>(*stream_id)] = -1;
    return QKV_OK;
}

int qkv_stream_close(qkv_handle *h, int32_t stream_id) {
    if (!h) return QKV_ERR_INVALID_ARG;
    // In-flight work may still read this stream's page-table row.
    CK(cudaSetDevice(h->device));
    CK(cudaStreamSynchronize(h->stream));
    std::string e;
    const std::vector<int32_t> *pg = h->pager->pages(stream_id);
    const size_t used = pg ? pg->size() : 0;
    const int rc = h->pager->close(stream_id, &e);
    if (rc) return fail(h, rc, e);
    int *row = h->h_page_table + static_cast<size_t>(stream_id) * h->maxp;
    std::fill(row, row + used, -1);
    CK(cudaMemcpyAsync(h->d_page_table + static_cast<size_t>(stream_id) * h->maxp, row, used * sizeof(int),
                       cudaMemcpyHostToDevice, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return QKV_OK;
}

int qkv_stream_length(const qkv_handle *h, int32_t stream_id, int32_t *tokens) {
    if (!h || !tokens) return QKV_ERR_INVALID_ARG;
    return h->pager->length(stream_id, tokens, nullptr);
}

int qkv_pool_stats(const qkv_handle *h, int64_t *free_pages, int64_t *total_pages) {
    if (!h) return QKV_ERR_INVALID_ARG;
    if (free_pages) *free_pages = h->pager->free_pages();
    if (total_pages) *total_pages = h->n_pages;
    return QKV_OK;
}

int qkv_compact(qkv_handle *h, int64_t *moved) {
    const TraceRange trace("qkv_compact");
    if (!h) return QKV_ERR_INVALID_ARG;
    CK(cudaSetDevice(h->device));
    CK(cudaStreamSynchronize(h->stream));
    std::vector<int32_t> src, dst;
    h->pager->compact(&src, &dst);
    if (moved) *moved = static_cast<int64_t>(src.size());
    if (!src.empty()) {
        DeviceTemp moves;
        CK(cudaMalloc(&moves.p, 2 * src.size() * sizeof(int)));
        int *d_moves = static_cast<int *>(moves.p);
        CK(cudaMemcpy(d_moves, src.data(), src.size() * sizeof(int), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(d_moves + src.size(), dst.data(), dst.size() * sizeof(int), cudaMemcpyHostToDevice));
        for (int l = 0; l < h->cfg.n_layers; ++l) {
            CK(launch_page_copy(static_cast<uint8_t *>(h->pool) + h->pool_layer_bytes * static_cast<size_t>(l),
                                h->page_bytes, d_moves, d_moves + src.size(), static_cast<int>(src.size()), h->stream));
            if (h->scales) {
                CK(launch_page_copy(h->scales + h->scales_layer_elems * static_cast<size_t>(l), kPageScales * sizeof(float),
                                    d_moves, d_moves + src.size(), static_cast<int>(src.size()), h->stream));
            }
        }
        CK(cudaStreamSynchronize(h->stream));
    }
    // Rewrite the whole page table from the pager.
    std::fill(h->h_page_table, h->h_page_table + static_cast<size_t>(h->rt.max_streams) * h->maxp, -1);
    for (int s = 0; s < h->rt.max_streams; ++s) {
        const std::vector<int32_t> *pg = h->pager->pages(s);
        if (!pg) continue;
        std::copy(pg->begin(), pg->end(), h->h_page_table + static_cast<size_t>(s) * h->maxp);
    }
    CK(cudaMemcpyAsync(h->d_page_table, h->h_page_table, static_cast<size_t>(h->rt.max_streams) * h->maxp * sizeof(int),
                       cudaMemcpyHostToDevice, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return QKV_OK;
}

// Decoder input from prompt ids (the device side of
// src/decoder-input.cpp:64-98).  Checks, per stream and in the reference's
// order: every id inside the embedding table, no more placeholders than the
// stream's audio rows, and as many.  Then row t of x is the embedding row of
// ids[t], or the stream's next audio row where ids[t] == audio_token_id.
// Audio rows in host memory go up through the pinned chunks into h->qkv
// (free until the first projection of a prefill writes it); rows already on
// the device are read where they are.
static int decoder_input_check(qkv_handle *h, int n, const int32_t *lens, const int32_t *ids,
                               const int32_t *audio_tokens, int32_t audio_token_id) {
    if (!lens || !ids || !audio_tokens) return fail(h, QKV_ERR_INVALID_ARG, "null lens, ids or audio_tokens");
    if (audio_token_id < 0) return fail(h, QKV_ERR_INVALID_ARG, "invalid decoder input configuration");
    size_t t = 0;
    for (int i = 0; i < n; ++i) {
        if (lens[i] <= 0) return fail(h, QKV_ERR_INVALID_ARG, "prompt length must be positive");
        if (audio_tokens[i] < 0) return fail(h, QKV_ERR_INVALID_ARG, "invalid native audio encoder output");
        int audio_positions = 0;
        for (int k = 0; k < lens[i]; ++k, ++t) {
            const int32_t id = ids[t];
            if (id < 0 || id >= h->cfg.vocab)
                return fail(h, QKV_ERR_INVALID_ARG, "decoder input token id is out of embedding range");
            if (id == audio_token_id) {
                if (audio_positions >= audio_tokens[i])
                    return fail(h, QKV_ERR_INVALID_ARG, "prompt has more audio placeholders than audio encoder outputs");
                ++audio_positions;
            }
        }
        if (audio_positions != audio_tokens[i])
            return fail(h, QKV_ERR_INVALID_ARG, "audio placeholder count does not match audio encoder output count");
    }
    return QKV_OK;
}

static int decoder_input_run(qkv_handle *h, int n, const int32_t *lens, const int32_t *ids,
                             const float *const *audio, const int32_t *audio_tokens, bool audio_on_device,
                             int32_t audio_token_id, float *x, cudaStream_t st) {
    const int H = h->cfg.hidden;
    int T = 0, A = 0;
    for (int i = 0; i < n; ++i) {
        T += lens[i];
        A += audio_tokens[i];
        if (audio_tokens[i] > 0 && (!audio || !audio[i]))
            return fail(h, QKV_ERR_INVALID_ARG, "null audio rows for a stream with audio placeholders");
    }
    if (T > h->max_rows) return fail(h, QKV_ERR_CAPACITY, "prompt tokens exceed max_batch_tokens");
    if (A > 0 && !audio_on_device && H > kQkvDim)
        return fail(h, QKV_ERR_STATE, "audio staging: hidden wider than the projection scratch");
    CK(cudaEventSynchronize(h->dec_ev));   // the pinned staging is free again
    int *hid = h->h_dec, *hsrc = h->h_dec + T;
    const float **hptr = h->h_rowptr;
    int t = 0, a = 0;
    for (int i = 0; i < n; ++i) {
        int k_audio = 0;
        for (int k = 0; k < lens[i]; ++k, ++t) {
            hid[t] = ids[t];
            if (ids[t] == audio_token_id) {
                hsrc[t] = a;
                hptr[a] = audio_on_device ? audio[i] + static_cast<size_t>(k_audio) * H
                                          : h->qkv + static_cast<size_t>(a) * H;
                ++a;
                ++k_audio;
            } else {
                hsrc[t] = -1;
            }
        }
    }
    int rc;
    if (A > 0 && !audio_on_device) {
        std::vector<const float *> blocks;
        std::vector<int32_t> counts;
        for (int i = 0; i < n; ++i) {
            if (audio_tokens[i] > 0) {
                blocks.push_back(audio[i]);
                counts.push_back(audio_tokens[i]);
            }
        }
        if ((rc = upload_prompt_rows(h, h->qkv, static_cast<int>(blocks.size()), blocks.data(), counts.data(), H, st)))
            return rc;
    }
    CK(cudaMemcpyAsync(h->d_dec, h->h_dec, 2 * static_cast<size_t>(T) * sizeof(int), cudaMemcpyHostToDevice, st));
    if (A > 0)
        CK(cudaMemcpyAsync(h->d_rowptr, h->h_rowptr, static_cast<size_t>(A) * sizeof(float *), cudaMemcpyHostToDevice,
                           st));
    CK(cudaEventRecord(h->dec_ev, st));
    CK(launch_decoder_input(h->d_dec, h->d_dec + T, T, h->embd, h->w_dtype, H, h->d_rowptr, x, st));
    h->launches += 1;
    return QKV_OK;
}

// Shared body of qkv_prefill (one contiguous embedding block) and
// qkv_prefill_rows (one block per stream): rows[i] = stream i's prompt rows.
static int prefill_impl(qkv_handle *h, int32_t n, const int32_t *stream_ids, const int32_t *lens,
                        const std::function<int()> &fill_x, int32_t *out_ids, float *out_logits) {
    int rc;
    if ((rc = check_streams(h, n, stream_ids))) return rc;
    int64_t total = 0;
    for (int i = 0; i < n; ++i) {
        if (lens[i] <= 0) return fail(h, QKV_ERR_INVALID_ARG, "prompt length must be positive");
        if (stream_len(h, stream_ids[i]) + static_cast<int64_t>(lens[i]) > h->rt.max_context)
            return fail(h, QKV_ERR_CAPACITY, "prompt exceeds max_context");
        total += lens[i];
    }
    if (total > h->max_rows) return fail(h, QKV_ERR_CAPACITY, "prompt tokens exceed max_batch_tokens");
    CK(cudaSetDevice(h->device));
    const int T = static_cast<int>(total);
    int *hs = row_stage(h), *hp = hs + T, *hr = hp + T;   // slots, positions, last-row indices
    int t = 0;
    for (int i = 0; i < n; ++i) {
        const int base = stream_len(h, stream_ids[i]);
        for (int k = 0; k < lens[i]; ++k, ++t) {
            hs[t] = stream_ids[i];
            hp[t] = base + k;
        }
        hr[i] = t - 1;
    }
    if ((rc = grow_streams(h, n, stream_ids, lens, h->stream))) return rc;
    int *ds = h->d_rowbuf, *dp = ds + T, *dr = dp + T;
    if ((rc = row_upload(h, hs, static_cast<size_t>(2 * T + n), h->stream))) return rc;
    if ((rc = fill_x())) return rc;
    int n_items = 0;
    std::vector<int> base(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i) base[static_cast<size_t>(i)] = hp[t_first(i, lens)];
    if ((rc = upload_items(h, n, lens, base.data(), &n_items, h->stream))) return rc;
    if ((rc = run_layers(h, T, ds, dp, nullptr, true, 0, -1, h->d_items, n_items))) return rc;
    if ((rc = head_and_argmax(h, n, dr))) return rc;
    return finish_ids(h, n, stream_ids, out_ids, out_logits);
}

int qkv_prefill(qkv_handle *h, int32_t n, const int32_t *stream_ids, const int32_t *lens, const float *embeddings,
                int32_t *out_ids, float *out_logits) {
    const TraceRange trace("qkv_prefill");
    if (!h) return QKV_ERR_INVALID_ARG;
    if (!h->has_weights) return fail(h, QKV_ERR_STATE, "handle has no model weights");
    if (!lens || !embeddings) return fail(h, QKV_ERR_INVALID_ARG, "null lens or embeddings");
    if (n < 0) return fail(h, QKV_ERR_INVALID_ARG, "negative stream count");
    std::vector<const float *> rows(static_cast<size_t>(n));
    size_t off = 0;
    for (int i = 0; i < n; ++i) {
        rows[static_cast<size_t>(i)] = embeddings + off;
        off += static_cast<size_t>(lens[i] > 0 ? lens[i] : 0) * h->cfg.hidden;
    }
    return prefill_impl(h, n, stream_ids, lens,
                        [&]() { return upload_prompt_rows(h, h->x, n, rows.data(), lens, h->cfg.hidden, h->stream); },
                        out_ids, out_logits);
}

int qkv_prefill_rows(qkv_handle *h, int32_t n, const int32_t *stream_ids, const int32_t *lens,
                     const float *const *embeddings, int32_t *out_ids, float *out_logits) {
    const TraceRange trace("qkv_prefill_rows");
    if (!h) return QKV_ERR_INVALID_ARG;
    if (!h->has_weights) return fail(h, QKV_ERR_STATE, "handle has no model weights");
    if (!lens || !embeddings) return fail(h, QKV_ERR_INVALID_ARG, "null lens or embeddings");
    for (int i = 0; i < n; ++i)
        if (!embeddings[i]) return fail(h, QKV_ERR_INVALID_ARG, "null embedding rows for a stream");
    return prefill_impl(h, n, stream_ids, lens,
                        [&]() { return upload_prompt_rows(h, h->x, n, embeddings, lens, h->cfg.hidden, h->stream); },
                        out_ids, out_logits);
}

int qkv_prefill_ids(qkv_handle *h, int32_t n, const int32_t *stream_ids, const int32_t *lens, const int32_t *ids,
                    const float *const *audio, const int32_t *audio_tokens, int32_t audio_on_device,
                    int32_t audio_token_id, int32_t *out_ids, float *out_logits) {
    const TraceRange trace("qkv_prefill_ids");
    if (!h) return QKV_ERR_INVALID_ARG;
    if (!h->has_weights) return fail(h, QKV_ERR_STATE, "handle has no model weights");
    if (n < 0) return fail(h, QKV_ERR_INVALID_ARG, "negative stream count");
    int rc;
    if ((rc = decoder_input_check(h, n, lens, ids, audio_tokens, audio_token_id))) return rc;
    return prefill_impl(h, n, stream_ids, lens,
                        [&]() {
                            return decoder_input_run(h, n, lens, ids, audio, audio_tokens, audio_on_device != 0,
                                                     audio_token_id, h->x, h->stream);
                        },
                        out_ids, out_logits);
}

int qkv_audio_projector_width(const qkv_handle *h, int32_t *width) {
    if (!h || !width) return QKV_ERR_INVALID_ARG;
    *width = h->audio_hidden;
    return QKV_OK;
}

// Audio projector (audio-encoder.cpp:848-856): LayerNorm -> proj0 + bias ->
// erf GELU -> proj1 + bias, rows of the audio encoder's output (device) to
// decoder-width rows (device).  Intermediates live in the handle's prefill
// scratch: LayerNorm output in act, proj0 sums in gu, GELU output in xn.
int qkv_audio_project(qkv_handle *h, int32_t n, const float *audio_dev, float *out_dev, void *stream) {
    const TraceRange trace("qkv_audio_project");
    if (!h) return QKV_ERR_INVALID_ARG;
    if (!h->has_weights || h->audio_hidden <= 0) return fail(h, QKV_ERR_STATE, "the model file has no audio projector");
    if (n < 0 || (n > 0 && (!audio_dev || !out_dev))) return fail(h, QKV_ERR_INVALID_ARG, "bad row count or pointer");
    if (n == 0) return QKV_OK;
    const int A = h->audio_hidden, H = h->cfg.hidden;
    if (n > h->max_rows) return fail(h, QKV_ERR_CAPACITY, "audio rows exceed max_batch_tokens");
    if (A > h->cfg.intermediate || A > H)
        return fail(h, QKV_ERR_STATE, "audio projector wider than the handle's row scratch");
    CK(cudaSetDevice(h->device));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const cudaStream_t saved = h->stream;   // the GEMM helper launches on h->stream
    h->stream = st;
    int rc = QKV_OK;
    cudaError_t e = launch_layernorm(audio_dev, n, A, h->ap_norm_w, h->ap_norm_b, 1.0e-5f, h->act, h->act_dtype, st);
    if (e == cudaSuccess) e = gemm(h, h->act, h->ap_w0, h->gu, n, A, A, 0);
    if (e == cudaSuccess) e = launch_bias_act(h->gu, h->ap_b0, n, A, true, h->xn, h->act_dtype, st);
    if (e == cudaSuccess) e = gemm(h, h->xn, h->ap_w1, out_dev, n, H, A, 0);
    if (e == cudaSuccess) e = launch_bias_act(out_dev, h->ap_b1, n, H, false, out_dev, kActF32, st);
    h->stream = saved;
    if (e != cudaSuccess) rc = cuda_fail(h, e, "audio projector");
    else h->launches += 5;
    return rc;
}

int qkv_decoder_input(qkv_handle *h, int32_t n, const int32_t *lens, const int32_t *ids, const float *const *audio,
                      const int32_t *audio_tokens, int32_t audio_on_device, int32_t audio_token_id, float *x_dev,
                      void *stream) {
    const TraceRange trace("qkv_decoder_input");
    if (!h) return QKV_ERR_INVALID_ARG;
    if (!h->has_weights) return fail(h, QKV_ERR_STATE, "handle has no model weights");
    if (n < 0 || !x_dev) return fail(h, QKV_ERR_INVALID_ARG, "negative stream count or null output");
    int rc;
    if ((rc = decoder_input_check(h, n, lens, ids, audio_tokens, audio_token_id))) return rc;
    CK(cudaSetDevice(h->device));
    return decoder_input_run(h, n, lens, ids, audio, audio_tokens, audio_on_device != 0, audio_token_id, x_dev,
                             static_cast<cudaStream_t>(stream));
}

int qkv_decode_step(qkv_handle *h, int32_t n, const int32_t *stream_ids, const int32_t *in_ids, int32_t *out_ids,
                    float *out_logits) {
    const TraceRange trace("qkv_decode_step");
    if (!h) return QKV_ERR_INVALID_ARG;
    if (!h->has_weights) return fail(h, QKV_ERR_STATE, "handle has no model weights");
    int rc;
    if ((rc = check_streams(h, n, stream_ids))) return rc;
    if (n > kAttnMaxRows) return fail(h, QKV_ERR_CAPACITY, "decode batch larger than 1024 rows");
    int *hs = row_stage(h), *hp = hs + n, *hl = hp + n, *hi = hl + n;
    for (int i = 0; i < n; ++i) {
        const int len = stream_len(h, stream_ids[i]);
        if (len <= 0) return fail(h, QKV_ERR_STATE, "decode on a stream with no prompt");
        if (len + 1 > h->rt.max_context) return fail(h, QKV_ERR_CAPACITY, "stream reached max_context");
        const int id = in_ids ? in_ids[i] : h->last_id[static_cast<size_t>(stream_ids[i])];
        if (id < 0 || id >= h->cfg.vocab) return fail(h, QKV_ERR_INVALID_ARG, "input id out of range");
        hs[i] = stream_ids[i];
        hp[i] = len;
        hl[i] = len + 1;
        hi[i] = id;
    }
    CK(cudaSetDevice(h->device));
    if ((rc = grow_streams(h, n, stream_ids, nullptr, h->stream))) return rc;
    int *ds = h->d_rowbuf, *dp = ds + n, *dl = dp + n, *di = dl + n;
    if ((rc = row_upload(h, hs, static_cast<size_t>(4 * n), h->stream))) return rc;
    auto body = [&]() -> int {
        CK(launch_embed(di, n, h->embd, h->w_dtype, h->cfg.hidden, h->cfg.vocab, h->x, h->d_err, h->stream));
        h->launches += 1;
        int r;
        if ((r = run_layers(h, n, ds, dp, dl, false))) return r;
        return head_and_argmax(h, n, nullptr);
    };
    // Replay a captured graph for a steady batch; a batch whose size keeps
    // changing (continuous batching) runs eagerly rather than capturing per size.
    auto it = h->decode_graphs.find(n);
    const bool steady = n == h->last_decode_n;
    h->last_decode_n = n;
    if (h->use_graphs && (it != h->decode_graphs.end() || steady)) {
        if (it == h->decode_graphs.end()) {
            if (h->decode_graphs.size() >= 32) {
                CK(cudaStreamSynchronize(h->stream));
                for (auto &kv : h->decode_graphs) cudaGraphExecDestroy(kv.second.exec);
                h->decode_graphs.clear();
            }
            qkv_handle::Graph g;
            rc = capture_graph(h, body, &g);
            if (rc) return rc;
            it = h->decode_graphs.emplace(n, g).first;
        }
        CK(cudaGraphLaunch(it->second.exec, h->stream));
        h->launches += it->second.kernels;
    } else if ((rc = body())) {
        return rc;
    }
    return finish_ids(h, n, stream_ids, out_ids, out_logits);
}

int qkv_layer_forward(qkv_handle *h, int32_t layer, int32_t tokens, const float *x, float *out) {
    const TraceRange trace("qkv_layer_forward");
    if (!h) return QKV_ERR_INVALID_ARG;
    if (!h->has_weights) return fail(h, QKV_ERR_STATE, "handle has no model weights");
    if (layer < 0 || layer >= h->cfg.n_layers || tokens <= 0 || !x || !out)
        return fail(h, QKV_ERR_INVALID_ARG, "layer_forward: bad layer, token count or pointer");
    if (tokens > h->max_rows || tokens > h->rt.max_context) return fail(h, QKV_ERR_CAPACITY, "layer_forward: too many tokens");
    CK(cudaSetDevice(h->device));
    int32_t s = -1;
    int rc = qkv_stream_open(h, &s);
    if (rc) return rc;
    int *hs = row_stage(h), *hp = hs + tokens;
    for (int t = 0; t < tokens; ++t) {
        hs[t] = s;
        hp[t] = t;
    }
    rc = grow_streams(h, 1, &s, &tokens, h->stream);
    if (rc == QKV_OK) rc = row_upload(h, hs, static_cast<size_t>(2 * tokens), h->stream);
    if (rc == QKV_OK) {
        const size_t bytes = static_cast<size_t>(tokens) * h->cfg.hidden * sizeof(float);
        cudaError_t e = cudaMemcpyAsync(h->x, x, bytes, cudaMemcpyHostToDevice, h->stream);
        if (e != cudaSuccess) rc = cuda_fail(h, e, "layer_forward upload");
        int n_items = 0;
        if (rc == QKV_OK) rc = upload_items(h, 1, &tokens, nullptr, &n_items, h->stream);
        if (rc == QKV_OK)
            rc = run_layers(h, tokens, h->d_rowbuf, h->d_rowbuf + tokens, nullptr, true, layer, layer + 1, h->d_items,
                            n_items);
        if (rc == QKV_OK && h->res_pending.n > 0) {
            e = launch_residual_fold(h->x, tokens, h->cfg.hidden, h->res_pending, h->stream);
            h->res_pending = ResidualFold{};
            if (e != cudaSuccess) rc = cuda_fail(h, e, "layer_forward fold");
        }
        if (rc == QKV_OK) {
            e = cudaMemcpyAsync(out, h->x, bytes, cudaMemcpyDeviceToHost, h->stream);
            if (e != cudaSuccess) rc = cuda_fail(h, e, "layer_forward download");
        }
        if (rc == QKV_OK) rc = check_device_error(h);
    }
    const std::string keep = h->last_error;
    const int rc2 = qkv_stream_close(h, s);
    if (rc) {
        h->last_error = keep;
        return rc;
    }
    return rc2;
}

int qkv_generate(qkv_handle *h, const float *embeddings, int32_t tokens, int32_t max_new_tokens, const int32_t *stop_ids,
                 int32_t n_stop, int32_t *out_ids, int32_t *n_out, int32_t *stopped) {
    const TraceRange trace("qkv_generate");
    if (!h) return QKV_ERR_INVALID_ARG;
    if (n_out) *n_out = 0;
    if (stopped) *stopped = 0;
    if (max_new_tokens < 0) return fail(h, QKV_ERR_INVALID_ARG, "max_new_tokens must be non-negative");
    if (tokens <= 0 || !embeddings) return fail(h, QKV_ERR_INVALID_ARG, "invalid generation input");
    if (static_cast<int64_t>(tokens) + max_new_tokens > h->rt.max_context)
        return fail(h, QKV_ERR_CAPACITY, "generation exceeds KV-cache capacity");
    if (max_new_tokens == 0) return QKV_OK;
    if (!out_ids || (n_stop > 0 && !stop_ids)) return fail(h, QKV_ERR_INVALID_ARG, "out_ids or stop_ids is null");
    int32_t s = -1;
    int rc = qkv_stream_open(h, &s);
    if (rc) return rc;
    int32_t id = -1;
    rc = qkv_prefill(h, 1, &s, &tokens, embeddings, &id, nullptr);
    for (int step = 0; rc == QKV_OK && step < max_new_tokens; ++step) {
        out_ids[step] = id;
        if (n_out) *n_out = step + 1;
        bool stop = false;
        for (int k = 0; k < n_stop; ++k) stop = stop || id == stop_ids[k];
        if (stop) {
            if (stopped) *stopped = 1;
            break;
        }
        if (step + 1 >= max_new_tokens) break;
        rc = qkv_decode_step(h, 1, &s, &id, &id, nullptr);
    }
    const std::string keep = h->last_error;
    const int rc2 = qkv_stream_close(h, s);
    if (rc) {
        h->last_error = keep;
        return rc;
    }
    return rc2;
}

int qkv_kv_append(qkv_handle *h, int32_t layer, int32_t n, const int32_t *slots_dev, const int32_t *positions_dev,
                  const float *qkv_dev, float *q_out_dev, void *stream) {
    if (!h) return QKV_ERR_INVALID_ARG;
    if (layer < 0 || layer >= h->cfg.n_layers || n < 0 || (n > 0 && (!slots_dev || !positions_dev || !qkv_dev || !q_out_dev)))
        return fail(h, QKV_ERR_INVALID_ARG, "kv_append: bad layer or pointer");
    CK(cudaSetDevice(h->device));
    cudaStream_t st = static_cast<cudaStream_t>(stream);   // NULL: the legacy default stream
    const qkv_handle::Layer &L = h->layers[static_cast<size_t>(layer)];
    AppendParams ap = append_params(h, layer, n, slots_dev, positions_dev, qkv_dev, q_out_dev, L.q_norm, L.k_norm);
    CK(launch_kv_append(ap, h->rt.kv_dtype, st));
    h->launches += 1;
    return QKV_OK;
}

int qkv_kv_attend(qkv_handle *h, int32_t layer, int32_t n, const int32_t *slots_dev, const int32_t *lens_dev,
                  const float *q_dev, float *out_dev, void *stream) {
    if (!h) return QKV_ERR_INVALID_ARG;
    if (layer < 0 || layer >= h->cfg.n_layers || n < 0 || n > kAttnMaxRows ||
        (n > 0 && (!slots_dev || !lens_dev || !q_dev || !out_dev)))
        return fail(h, QKV_ERR_INVALID_ARG, "kv_attend: bad layer, row count or pointer");
    CK(cudaSetDevice(h->device));
    cudaStream_t st = static_cast<cudaStream_t>(stream);   // NULL: the legacy default stream
    AttendParams at = attend_params(h, layer, n, slots_dev, lens_dev, q_dev, out_dev);
    CK(launch_decode_attn(at, h->rt.kv_dtype, false, h->num_sms, st));
    h->launches += 1;
    return QKV_OK;
}

// Shared body of the two prefill-attention operators: exactly one of q (f32)
// and q16 (K3's operand form) is given.
static int prefill_attend_op(qkv_handle *h, int32_t layer, int32_t n, const int32_t *stream_ids, const int32_t *lens,
                      const float *q, const void *q16, float *out, void *stream) {
    if (!h) return QKV_ERR_INVALID_ARG;
    if (layer < 0 || layer >= h->cfg.n_layers || n < 0 || (n > 0 && (!stream_ids || !lens || !(q || q16) || !out)))
        return fail(h, QKV_ERR_INVALID_ARG, "prefill_attend: bad layer, count or pointer");
    if (q16 && !(h->prefill_tc && prefill_tc_supported(h->rt.kv_dtype)))
        return fail(h, QKV_ERR_STATE, "prefill_attend_q16: needs a bf16 or 8-bit cache with the tensor-core kernel");
    int rc;
    if ((rc = check_streams(h, n, stream_ids))) return rc;
    int64_t total = 0;
    for (int i = 0; i < n; ++i) {
        if (lens[i] <= 0 || lens[i] > stream_len(h, stream_ids[i]))
            return fail(h, QKV_ERR_INVALID_ARG, "prefill_attend: query count must be in 1..stream length");
        total += lens[i];
    }
    if (total > h->max_rows) return fail(h, QKV_ERR_CAPACITY, "prefill_attend rows exceed max_batch_tokens");
    if (total == 0) return QKV_OK;
    CK(cudaSetDevice(h->device));
    cudaStream_t st = static_cast<cudaStream_t>(stream);   // NULL: the legacy default stream
    const int T = static_cast<int>(total);
    int *hs = row_stage(h), *hp = hs + T;
    int t = 0;
    for (int i = 0; i < n; ++i) {
        const int base = stream_len(h, stream_ids[i]) - lens[i];
        for (int k = 0; k < lens[i]; ++k, ++t) {
            hs[t] = stream_ids[i];
            hp[t] = base + k;
        }
    }
    if ((rc = row_upload(h, hs, static_cast<size_t>(2 * T), st))) return rc;
    int n_items = 0;
    std::vector<int> base(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i) base[static_cast<size_t>(i)] = stream_len(h, stream_ids[i]) - lens[i];
    if ((rc = upload_items(h, n, lens, base.data(), &n_items, st))) return rc;
    CK(prefill_attend(h, layer, T, h->d_rowbuf, h->d_rowbuf + T, q, q16, out, false, h->d_items, n_items, st));
    h->launches += (!q16 && prefill_on_tc(h, h->d_items, n_items)) ? 2 : 1;
    return QKV_OK;
}

int qkv_prefill_attend(qkv_handle *h, int32_t layer, int32_t n, const int32_t *stream_ids, const int32_t *lens,
                       const float *q_dev, float *out_dev, void *stream) {
    return prefill_attend_op(h, layer, n, stream_ids, lens, q_dev, nullptr, out_dev, stream);
}

int qkv_prefill_attend_q16(qkv_handle *h, int32_t layer, int32_t n, const int32_t *stream_ids, const int32_t *lens,
                           const void *q16_dev, float *out_dev, void *stream) {
    return prefill_attend_op(h, layer, n, stream_ids, lens, nullptr, q16_dev, out_dev, stream);
}

int qkv_kv_step(qkv_handle *h, int32_t n, const int32_t *stream_ids, const float *qkv_dev, float *out_dev, void *stream) {
    const TraceRange trace("qkv_kv_step");
    if (!h) return QKV_ERR_INVALID_ARG;
    int rc;
    if ((rc = check_streams(h, n, stream_ids))) return rc;
    if (n > kAttnMaxRows) return fail(h, QKV_ERR_CAPACITY, "kv_step batch larger than 1024 rows");
    if (!qkv_dev || !out_dev) return fail(h, QKV_ERR_INVALID_ARG, "null device pointer");
    CK(cudaSetDevice(h->device));
    cudaStream_t st = static_cast<cudaStream_t>(stream);   // NULL: the legacy default stream
    int *hs = row_stage(h), *hp = hs + n, *hl = hp + n;
    for (int i = 0; i < n; ++i) {
        const int len = stream_len(h, stream_ids[i]);
        if (len + 1 > h->rt.max_context) return fail(h, QKV_ERR_CAPACITY, "stream reached max_context");
        hs[i] = stream_ids[i];
        hp[i] = len;
        hl[i] = len + 1;
    }
    if ((rc = grow_streams(h, n, stream_ids, nullptr, st))) return rc;
    int *ds = h->d_rowbuf, *dp = ds + n, *dl = dp + n;
    if ((rc = row_upload(h, hs, static_cast<size_t>(3 * n), st))) return rc;
    const size_t in_stride = static_cast<size_t>(n) * kQkvDim, out_stride = static_cast<size_t>(n) * kQDim;
    auto body = [&](cudaStream_t on) -> int {
        const int L = h->cfg.n_layers;
        for (int l = 0; l < L; ++l) {
            int r;
            if ((r = kv_step_layer(h, l, n, ds, dp, dl, qkv_dev + in_stride * l,
                                   l + 1 < L ? qkv_dev + in_stride * (l + 1) : nullptr, out_dev + out_stride * l, on)))
                return r;
        }
        return QKV_OK;
    };
    if (!h->use_graphs) return body(st);
    const auto key = std::make_tuple(n, static_cast<const void *>(qkv_dev), static_cast<const void *>(out_dev));
    auto it = h->kv_graphs.find(key);
    if (it == h->kv_graphs.end()) {
        if (h->kv_graphs.size() >= 64) {
            CK(cudaDeviceSynchronize());
            for (auto &kv : h->kv_graphs) cudaGraphExecDestroy(kv.second.exec);
            h->kv_graphs.clear();
        }
        qkv_handle::Graph g;
        rc = capture_graph(h, [&]() { return body(h->stream); }, &g);
        if (rc) return rc;
        it = h->kv_graphs.emplace(key, g).first;
    }
    CK(cudaGraphLaunch(it->second.exec, st));
    h->launches += it->second.kernels;
    return QKV_OK;
}

// Host-buffer KV step, pipelined by layer: layer l's inputs go up on
// copy_in a few layers ahead of their use (paced by the attention kernels),
// layer l's kernels wait only for the inputs they read (their own, and layer
// l + 1's with the append-ahead), and layer l's outputs come back on
// copy_out as soon as its attention has run, so PCIe traffic in both
// directions overlaps the kernels.
int qkv_kv_step_host(qkv_handle *h, int32_t n, const int32_t *stream_ids, const float *qkv_host, float *out_host) {
    const TraceRange trace("qkv_kv_step_host");
    if (!h) return QKV_ERR_INVALID_ARG;
    if (!qkv_host || !out_host || n <= 0) return fail(h, QKV_ERR_INVALID_ARG, "null host pointer or empty batch");
    int rc;
    if ((rc = check_streams(h, n, stream_ids))) return rc;
    if (n > kAttnMaxRows) return fail(h, QKV_ERR_CAPACITY, "kv_step batch larger than 1024 rows");
    CK(cudaSetDevice(h->device));
    const int L = h->cfg.n_layers;
    const size_t in_stride = static_cast<size_t>(n) * kQkvDim, out_stride = static_cast<size_t>(n) * kQDim;
    const size_t in_elems = in_stride * L, out_elems = out_stride * L;
    const size_t need = (in_elems + out_elems) * sizeof(float);
    if (need > h->host_stage_bytes) {   // device staging, grown on demand and kept
        CK(cudaDeviceSynchronize());
        for (auto &kv : h->kvh_graphs) cudaGraphExecDestroy(kv.second.exec);
        h->kvh_graphs.clear();
        cudaFree(h->host_stage);
        h->host_stage = nullptr;
        h->host_stage_bytes = 0;
        CK(cudaMalloc(&h->host_stage, need));
        h->host_stage_bytes = need;
    }
    if (!h->copy_in) {
        CK(cudaStreamCreateWithFlags(&h->copy_in, cudaStreamNonBlocking));
        CK(cudaStreamCreateWithFlags(&h->copy_out, cudaStreamNonBlocking));
        CK(cudaEventCreateWithFlags(&h->ev_tail, cudaEventDisableTiming));
    }
    while (static_cast<int>(h->ev_in.size()) < L) {
        cudaEvent_t a = nullptr, b = nullptr;
        CK(cudaEventCreateWithFlags(&a, cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&b, cudaEventDisableTiming));
        h->ev_in.push_back(a);
        h->ev_done.push_back(b);
    }
    float *stage_in = h->host_stage, *stage_out = h->host_stage + in_elems;
    // Rows: as qkv_kv_step (one appended token per stream).
    int *hs = row_stage(h), *hp = hs + n, *hl = hp + n;
    for (int i = 0; i < n; ++i) {
        const int len = stream_len(h, stream_ids[i]);
        if (len + 1 > h->rt.max_context) return fail(h, QKV_ERR_CAPACITY, "stream reached max_context");
        hs[i] = stream_ids[i];
        hp[i] = len;
        hl[i] = len + 1;
    }
    if ((rc = grow_streams(h, n, stream_ids, nullptr, h->stream))) return rc;
    int *ds = h->d_rowbuf, *dp = ds + n, *dl = dp + n;
    if ((rc = row_upload(h, hs, static_cast<size_t>(3 * n), h->stream))) return rc;
    // The staging is free once the work queued so far on h->stream has run
    // (earlier calls' kernels and output copies end there).
    // Uploads are paced: the first kAhead layers' inputs go up at once, then
    // layer l + kAhead's once layer l's attention has finished.  Sent back to
    // back, the 28 uploads (4.2 MB each at config 4) overlap the first layers'
    // attention at full PCIe rate and slow it far more than the same bytes
    // spread over the step do (measured: +2.3 ms per step against +0.2 ms).
    constexpr int kAhead = 4;
    auto upload = [&](int l) -> int {
        CK(cudaMemcpyAsync(stage_in + in_stride * l, qkv_host + in_stride * l, in_stride * sizeof(float),
                           cudaMemcpyHostToDevice, h->copy_in));
        CK(cudaEventRecord(h->ev_in[static_cast<size_t>(l)], h->copy_in));
        return QKV_OK;
    };
    auto body = [&]() -> int {
        CK(cudaEventRecord(h->ev_tail, h->stream));
        CK(cudaStreamWaitEvent(h->copy_in, h->ev_tail, 0));
        int r = QKV_OK;
        for (int l = 0; l < L && l < kAhead; ++l)
            if ((r = upload(l))) return r;
        for (int l = 0; l < L; ++l) {
            CK(cudaStreamWaitEvent(h->stream, h->ev_in[static_cast<size_t>(l)], 0));
            // With the append-ahead, layer l's launch (from layer 1 on: layer 0's
            // attention starts on layer 0's inputs alone) also reads layer l + 1's.
            if (h->append_ahead && l >= 1 && l + 1 < L)
                CK(cudaStreamWaitEvent(h->stream, h->ev_in[static_cast<size_t>(l + 1)], 0));
            if ((r = kv_step_layer(h, l, n, ds, dp, dl, stage_in + in_stride * l,
                                   l + 1 < L ? stage_in + in_stride * (l + 1) : nullptr, stage_out + out_stride * l,
                                   h->stream, 1)))
                break;
            CK(cudaEventRecord(h->ev_done[static_cast<size_t>(l)], h->stream));
            CK(cudaStreamWaitEvent(h->copy_out, h->ev_done[static_cast<size_t>(l)], 0));
            CK(cudaMemcpyAsync(out_host + out_stride * l, stage_out + out_stride * l, out_stride * sizeof(float),
                               cudaMemcpyDeviceToHost, h->copy_out));
            if (l + kAhead < L) {
                CK(cudaStreamWaitEvent(h->copy_in, h->ev_done[static_cast<size_t>(l)], 0));
                if ((r = upload(l + kAhead))) break;
            }
        }
        // Every copy of this call has run before the stream's later work.
        CK(cudaEventRecord(h->ev_tail, h->copy_out));
        CK(cudaStreamWaitEvent(h->stream, h->ev_tail, 0));
        CK(cudaEventRecord(h->ev_tail, h->copy_in));
        CK(cudaStreamWaitEvent(h->stream, h->ev_tail, 0));
        return r;
    };
    // Pinned host buffers: the whole sequence (copies on both copy streams,
    // kernels, the events between them) replays as one graph, which also keeps
    // the programmatic launch edges between consecutive attention kernels that
    // eager event waits and records in the stream would cut.  Pageable
    // buffers take the eager path (their copies cannot be captured).
    cudaPointerAttributes ai{}, ao{};
    const bool pinned = cudaPointerGetAttributes(&ai, qkv_host) == cudaSuccess && ai.type == cudaMemoryTypeHost &&
                        cudaPointerGetAttributes(&ao, out_host) == cudaSuccess && ao.type == cudaMemoryTypeHost;
    (void)cudaGetLastError();   // an unregistered pointer may leave an error behind on older drivers
    if (h->use_graphs && pinned) {
        const auto key = std::make_tuple(n, static_cast<const void *>(qkv_host), static_cast<const void *>(out_host),
                                         static_cast<const void *>(h->host_stage));
        auto it = h->kvh_graphs.find(key);
        if (it == h->kvh_graphs.end()) {
            if (h->kvh_graphs.size() >= 16) {
                CK(cudaDeviceSynchronize());
                for (auto &kv : h->kvh_graphs) cudaGraphExecDestroy(kv.second.exec);
                h->kvh_graphs.clear();
            }
            qkv_handle::Graph g;
            if ((rc = capture_graph(h, body, &g))) return rc;
            it = h->kvh_graphs.emplace(key, g).first;
        }
        CK(cudaGraphLaunch(it->second.exec, h->stream));
        h->launches += it->second.kernels;
    } else {
        rc = body();
    }
    const int rc2 = check_device_error(h);
    return rc ? rc : rc2;
}

int qkv_stream_extend(qkv_handle *h, int32_t stream_id, int32_t tokens) {
    if (!h) return QKV_ERR_INVALID_ARG;
    if (tokens < 0) return fail(h, QKV_ERR_INVALID_ARG, "tokens must be non-negative");
    if (!h->pager->is_open(stream_id)) return fail(h, QKV_ERR_INVALID_ARG, "stream is not open");
    if (stream_len(h, stream_id) + static_cast<int64_t>(tokens) > h->rt.max_context)
        return fail(h, QKV_ERR_CAPACITY, "extend exceeds max_context");
    CK(cudaSetDevice(h->device));
    int rc = grow_streams(h, 1, &stream_id, &tokens, h->stream);
    if (rc) return rc;
    CK(cudaStreamSynchronize(h->stream));
    return QKV_OK;
}

int qkv_fill_random(qkv_handle *h, uint64_t seed) {
    if (!h) return QKV_ERR_INVALID_ARG;
    CK(cudaSetDevice(h->device));
    std::vector<int> pages;
    for (int s = 0; s < h->rt.max_streams; ++s) {
        const std::vector<int32_t> *pg = h->pager->pages(s);
        if (pg) pages.insert(pages.end(), pg->begin(), pg->end());
    }
    if (pages.empty()) return QKV_OK;
    DeviceTemp list;
    CK(cudaMalloc(&list.p, pages.size() * sizeof(int)));
    int *d = static_cast<int *>(list.p);
    CK(cudaMemcpy(d, pages.data(), pages.size() * sizeof(int), cudaMemcpyHostToDevice));
    for (int l = 0; l < h->cfg.n_layers; ++l) {
        CK(launch_page_fill(static_cast<uint8_t *>(h->pool) + h->pool_layer_bytes * static_cast<size_t>(l),
                            h->scales ? h->scales + h->scales_layer_elems * static_cast<size_t>(l) : nullptr,
                            h->rt.kv_dtype, d, static_cast<int>(pages.size()), seed * 1000003ull + static_cast<uint64_t>(l),
                            h->stream));
    }
    CK(cudaStreamSynchronize(h->stream));
    return QKV_OK;
}

int qkv_gather(qkv_handle *h, int32_t layer, int32_t stream_id, void *k_host, void *v_host, float *scales_out) {
    if (!h) return QKV_ERR_INVALID_ARG;
    if (layer < 0 || layer >= h->cfg.n_layers || !h->pager->is_open(stream_id) || !k_host || !v_host)
        return fail(h, QKV_ERR_INVALID_ARG, "gather: bad layer, stream or pointer");
    CK(cudaSetDevice(h->device));
    CK(cudaStreamSynchronize(h->stream));
    const int len = stream_len(h, stream_id);
    const std::vector<int32_t> *pg = h->pager->pages(stream_id);
    if (len == 0) return QKV_OK;
    const size_t eb = kv_elem_bytes(h->rt.kv_dtype);
    const size_t bytes = static_cast<size_t>(len) * kKvDim * eb;
    DeviceTemp target;
    CK(cudaMalloc(&target.p, 2 * bytes + pg->size() * sizeof(int)));
    uint8_t *d = static_cast<uint8_t *>(target.p);
    int *dpages = reinterpret_cast<int *>(d + 2 * bytes);
    CK(cudaMemcpy(dpages, pg->data(), pg->size() * sizeof(int), cudaMemcpyHostToDevice));
    CK(launch_page_gather(static_cast<uint8_t *>(h->pool) + h->pool_layer_bytes * static_cast<size_t>(layer),
                          h->rt.kv_dtype, dpages, static_cast<int>(pg->size()), len, h->n_pages, d, d + bytes, h->d_err,
                          h->stream));
    CK(cudaMemcpyAsync(k_host, d, bytes, cudaMemcpyDeviceToHost, h->stream));
    CK(cudaMemcpyAsync(v_host, d + bytes, bytes, cudaMemcpyDeviceToHost, h->stream));
    if (scales_out && h->scales) {
        for (size_t i = 0; i < pg->size(); ++i) {
            CK(cudaMemcpyAsync(scales_out + i * kPageScales,
                               h->scales + h->scales_layer_elems * static_cast<size_t>(layer) +
                                   static_cast<size_t>((*pg)[i]) * kPageScales,
                               kPageScales * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
        }
    }
    return check_device_error(h);
}

int qkv_stream_pages(const qkv_handle *h, int32_t stream_id, int32_t *pages_out, int32_t cap, int32_t *n) {
    if (!h || !n || (cap > 0 && !pages_out)) return QKV_ERR_INVALID_ARG;
    const std::vector<int32_t> *pg = h->pager->pages(stream_id);
    if (!pg) return QKV_ERR_INVALID_ARG;
    *n = static_cast<int32_t>(pg->size());
    for (int32_t i = 0; i < cap && i < *n; ++i) pages_out[i] = (*pg)[static_cast<size_t>(i)];
    return QKV_OK;
}

int qkv_page_read_probe(qkv_handle *h, int32_t layer, int32_t n, const int32_t *pages_dev, void *stream) {
    if (!h || n < 0 || (n > 0 && !pages_dev)) return QKV_ERR_INVALID_ARG;
    if (layer < 0 || layer >= h->cfg.n_layers) return fail(h, QKV_ERR_INVALID_ARG, "read probe: bad layer");
    if (h->page_bytes > 65536) return fail(h, QKV_ERR_STATE, "read probe: pages larger than 64 KB (f32 cache)");
    CK(cudaSetDevice(h->device));
    CK(launch_page_read_probe(static_cast<const uint8_t *>(h->pool) + h->pool_layer_bytes * static_cast<size_t>(layer),
                              static_cast<uint32_t>(h->page_bytes), pages_dev, n, h->n_pages, h->num_sms, h->d_err,
                              static_cast<cudaStream_t>(stream)));
    ++h->launches;
    return QKV_OK;
}

int qkv_debug_residual(qkv_handle *h, int32_t n, float *out) {
    if (!h || !out || n <= 0) return QKV_ERR_INVALID_ARG;
    if (!h->has_weights) return fail(h, QKV_ERR_STATE, "handle has no model weights");
    if (n > h->rt.max_streams) return fail(h, QKV_ERR_INVALID_ARG, "more rows than the decode batch can hold");
    CK(cudaSetDevice(h->device));
    CK(cudaMemcpyAsync(out, h->x, static_cast<size_t>(n) * h->cfg.hidden * sizeof(float), cudaMemcpyDeviceToHost,
                       h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return QKV_OK;
}

int qkv_debug_wait_timeout(qkv_handle *h, int64_t limit_cycles) {
    if (!h || limit_cycles < 1 || limit_cycles > qkv::kWaitLimitCycles) return QKV_ERR_INVALID_ARG;
    CK(cudaSetDevice(h->device));
    CK(launch_wait_probe(h->d_err, static_cast<long long>(limit_cycles), h->stream));
    ++h->launches;
    return QKV_OK;
}

int qkv_sync(qkv_handle *h) {
    if (!h) return QKV_ERR_INVALID_ARG;
    CK(cudaSetDevice(h->device));
    CK(cudaDeviceSynchronize());   // operator-level calls may run on any stream of this device
    return check_device_error(h);
}

int qkv_last_launches(const qkv_handle *h, int64_t *kernels) {
    if (!h || !kernels) return QKV_ERR_INVALID_ARG;
    *kernels = h->launches;
    return QKV_OK;
}

int qkv_gemm_bf16(const void *x, const void *w, float *c, int32_t m, int32_t n, int32_t k, int32_t accumulate,
                  void *stream) {
    if (!x || !w || !c || m < 0 || n < 0 || k <= 0 || k % 64 != 0) return QKV_ERR_INVALID_ARG;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return QKV_ERR_NO_DEVICE;
    static std::once_flag once;
    static cudaError_t prep = cudaSuccess;
    std::call_once(once, [] { prep = prepare_gemm_tc(); });
    if (prep != cudaSuccess) return QKV_ERR_CUDA;
    if (!gemm_tc_supported(m, n, k)) return QKV_ERR_INVALID_ARG;
    return launch_gemm_tc(x, w, c, m, n, k, accumulate ? 1 : 0, sms, nullptr, static_cast<cudaStream_t>(stream)) ==
                   cudaSuccess
               ? QKV_OK
               : QKV_ERR_CUDA;
}

int qkv_gemm_swiglu_bf16(const void *x, const void *w, void *act, int32_t m, int32_t n2, int32_t k, float *workspace,
                         int32_t *flags, int64_t workspace_floats, int32_t flag_tiles, void *stream) {
    if (!x || !w || !act || m < 0 || n2 < 0 || n2 % 2 != 0 || k <= 0 || k % 64 != 0) return QKV_ERR_INVALID_ARG;
    if ((workspace != nullptr) != (flags != nullptr) || workspace_floats < 0 || flag_tiles < 0) return QKV_ERR_INVALID_ARG;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return QKV_ERR_NO_DEVICE;
    static std::once_flag once;
    static cudaError_t prep = cudaSuccess;
    std::call_once(once, [] { prep = prepare_gemm_tc(); });
    if (prep != cudaSuccess) return QKV_ERR_CUDA;
    if (!gemm_tc_supported(m, n2, k)) return QKV_ERR_INVALID_ARG;
    return launch_gemm_tc_swiglu(x, w, act, m, n2, k, sms, nullptr, static_cast<cudaStream_t>(stream), workspace, flags,
                                 static_cast<size_t>(workspace_floats), flag_tiles) == cudaSuccess
               ? QKV_OK
               : QKV_ERR_CUDA;
}

int qkv_gemm_fp8(const void *x, const float *x_scale, const void *w, const float *w_scale, float *c, int32_t m, int32_t n,
                 int32_t k, int32_t accumulate, void *stream) {
    if (!x || !x_scale || !w || !w_scale || !c || m < 0 || n < 0 || k <= 0 || k % 128 != 0) return QKV_ERR_INVALID_ARG;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return QKV_ERR_NO_DEVICE;
    static std::once_flag once;
    static cudaError_t prep = cudaSuccess;
    std::call_once(once, [] { prep = prepare_gemm_tc(); });
    if (prep != cudaSuccess) return QKV_ERR_CUDA;
    if (!gemm_tc_fp8_supported(m, n, k)) return QKV_ERR_INVALID_ARG;
    return launch_gemm_tc_fp8(x, x_scale, w, w_scale, c, m, n, k, accumulate ? 1 : 0, sms, nullptr,
                              static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? QKV_OK
               : QKV_ERR_CUDA;
}

int qkv_quantize_rows_e4m3(const void *x_bf16, int32_t rows, int32_t k, void *codes, float *scales, void *stream) {
    if (!x_bf16 || !codes || !scales || rows < 0 || k <= 0 || k % 4 != 0 || k > rows_q8_max_k())
        return QKV_ERR_INVALID_ARG;
    return launch_rows_q8(0, x_bf16, rows, k, nullptr, 0.0f, codes, scales, static_cast<cudaStream_t>(stream)) ==
                   cudaSuccess
               ? QKV_OK
               : QKV_ERR_CUDA;
}

int qkv_gguf_tensor(const char *gguf_path, const char *name, int64_t *ne_out, int32_t *n_dims, int32_t *ggml_type,
                    void *data_out, size_t cap_bytes, char *err, size_t err_len) {
    if (!name || !ne_out || !n_dims || !ggml_type) {
        set_err(err, err_len, "null argument");
        return QKV_ERR_INVALID_ARG;
    }
    GgufFile f;
    std::string e;
    const int rc = f.open(gguf_path, &e);
    if (rc) {
        set_err(err, err_len, e);
        return rc;
    }
    const GgufTensor *t = f.find(name);
    if (!t) {
        set_err(err, err_len, std::string("missing GGUF tensor: ") + name);
        return QKV_ERR_FORMAT;
    }
    for (int i = 0; i < 4; ++i) ne_out[i] = i < static_cast<int>(t->ne.size()) ? t->ne[static_cast<size_t>(i)] : 1;
    *n_dims = static_cast<int32_t>(t->ne.size());
    *ggml_type = static_cast<int32_t>(t->type);
    if (data_out && t->nbytes) std::memcpy(data_out, t->data, std::min(cap_bytes, t->nbytes));
    return QKV_OK;
}

// ---- host-only pager ----
qkv_pager *qkv_pager_create(int64_t n_pages, int32_t page_tokens, int32_t max_streams, int32_t max_pages_per_stream,
                            uint32_t seed) {
    if (n_pages <= 0 || n_pages > (int64_t{1} << 30) || page_tokens <= 0 || max_streams <= 0 || max_pages_per_stream <= 0)
        return nullptr;
    try {
        return reinterpret_cast<qkv_pager *>(new Pager(n_pages, page_tokens, max_streams, max_pages_per_stream, seed));
    } catch (const std::exception &) {
        return nullptr;   // the free list (4 bytes a page) does not fit in host memory
    }
}
void qkv_pager_destroy(qkv_pager *p) { delete reinterpret_cast<Pager *>(p); }
int qkv_pager_open(qkv_pager *p, int32_t *stream_id) {
    return p ? reinterpret_cast<Pager *>(p)->open(stream_id, nullptr) : QKV_ERR_INVALID_ARG;
}
int qkv_pager_close(qkv_pager *p, int32_t stream_id) {
    return p ? reinterpret_cast<Pager *>(p)->close(stream_id, nullptr) : QKV_ERR_INVALID_ARG;
}
int qkv_pager_append(qkv_pager *p, int32_t stream_id, int32_t tokens, int32_t *new_pages) {
    if (!p) return QKV_ERR_INVALID_ARG;
    if (new_pages) *new_pages = 0;
    try {
        std::vector<int32_t> added;
        const int rc = reinterpret_cast<Pager *>(p)->append(stream_id, tokens, &added, nullptr);
        if (new_pages && rc == QKV_OK) *new_pages = static_cast<int32_t>(added.size());
        return rc;
    } catch (const std::exception &) {
        return QKV_ERR_HOST_MEMORY;
    }
}
int qkv_pager_length(const qkv_pager *p, int32_t stream_id, int32_t *tokens) {
    return p ? reinterpret_cast<const Pager *>(p)->length(stream_id, tokens, nullptr) : QKV_ERR_INVALID_ARG;
}
int qkv_pager_pages(const qkv_pager *p, int32_t stream_id, int32_t *pages_out, int32_t cap, int32_t *n) {
    if (!p || !n || (cap > 0 && !pages_out)) return QKV_ERR_INVALID_ARG;
    const std::vector<int32_t> *pg = reinterpret_cast<const Pager *>(p)->pages(stream_id);
    if (!pg) return QKV_ERR_INVALID_ARG;
    *n = static_cast<int32_t>(pg->size());
    for (int32_t i = 0; i < cap && i < *n; ++i) pages_out[i] = (*pg)[static_cast<size_t>(i)];
    return QKV_OK;
}
int64_t qkv_pager_free_pages(const qkv_pager *p) { return p ? reinterpret_cast<const Pager *>(p)->free_pages() : -1; }
int qkv_pager_compact(qkv_pager *p, int32_t *src, int32_t *dst, int64_t cap, int64_t *n_moves) {
    if (!p) return QKV_ERR_INVALID_ARG;
    std::vector<int32_t> s, d;
    try {
        reinterpret_cast<Pager *>(p)->compact(&s, &d);
    } catch (const std::exception &) {
        return QKV_ERR_HOST_MEMORY;
    }
    if (n_moves) *n_moves = static_cast<int64_t>(s.size());
    for (int64_t i = 0; i < cap && i < static_cast<int64_t>(s.size()); ++i) {
        if (src) src[i] = s[static_cast<size_t>(i)];
        if (dst) dst[i] = d[static_cast<size_t>(i)];
    }
    return QKV_OK;
}
int qkv_pager_check(const qkv_pager *p) {
    return p ? reinterpret_cast<const Pager *>(p)->check(nullptr) : QKV_ERR_INVALID_ARG;
}

}  // extern "C"
