// extern "C" layer of include/quanta_b200.h over the engine and the ops-level kernels.
#include <cuda_runtime.h>

#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "quanta_b200.h"
#include "capi_util.h"
#include "engine.h"
#include "gemm_tc.h"
#include "ops.h"

struct qnt_dtensor {
    qb::DMat m;
    void* q = nullptr;
    void* d = nullptr;
    qb::TcMap wmap{};          // TMA source for the tensor-core matmul
    bool tc = false;           // wmap is valid
    void* tcbuf = nullptr;     // the copies wmap reads (stage-major scales; Q4_0: int8 q - 8)
    unsigned* status = nullptr;  // device status word of this tensor's kernels
};

struct qnt_model {
    qb::Engine eng;
};

namespace qnt_capi {

thread_local std::string g_err;

int set_err(int code, const std::string& m) {
    g_err = m;
    return code;
}

int cuda_err(cudaError_t e, const char* what) { return set_err(QNT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e)); }

}  // namespace qnt_capi

namespace {

using namespace qnt_capi;

int engine_code(qb::Engine& e, int r) {
    if (r >= 0) return r;
    g_err = e.error();
    switch (r) {
        case -2: return QNT_ERR_CUDA;
        case -4: return QNT_ERR_UNSUPPORTED;
        case -5: return QNT_ERR_RANGE;
        case -6: return QNT_ERR_DEVICE;
        default: return QNT_ERR_INVALID;
    }
}

bool shape_ok(int dtype, int rows, int cols) {
    return (dtype == QNT_Q8_0 || dtype == QNT_Q4_0) && rows > 0 && cols > 0 && cols % 32 == 0;
}

}  // namespace

extern "C" {

const char* qnt_last_error(void) { return qnt_capi::g_err.c_str(); }
int qnt_version(void) { return 100; }

int qnt_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

int qnt_set_device(int device) {
    cudaError_t e = cudaSetDevice(device);
    return e == cudaSuccess ? QNT_OK : cuda_err(e, "cudaSetDevice");
}

// ---------------------------------------------------------------- ops level

int qnt_tensor_upload(int dtype, int rows, int cols, const void* host_data, qnt_dtensor** out) {
    if (!out || !host_data || !shape_ok(dtype, rows, cols)) return set_err(QNT_ERR_INVALID, "bad tensor shape or dtype");
    auto t = std::make_unique<qnt_dtensor>();
    const size_t qbytes = size_t(rows) * qb::row_bytes_host(dtype, cols), sbytes = size_t(rows) * (cols / 32) * 2;
    cudaError_t e = cudaMalloc(&t->q, qbytes);
    if (e == cudaSuccess) e = cudaMalloc(&t->d, sbytes);
    if (e == cudaSuccess) e = cudaMemcpy(t->q, host_data, qbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(t->d, static_cast<const uint8_t*>(host_data) + qbytes, sbytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(t->q);
        cudaFree(t->d);
        return cuda_err(e, "tensor upload");
    }
    t->m.dtype = dtype;
    t->m.rows = rows;
    t->m.cols = cols;
    t->m.q = static_cast<const uint8_t*>(t->q);
    t->m.d = static_cast<const __half*>(t->d);
    e = cudaMalloc(&t->status, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(t->status, 0, sizeof(unsigned));
    if (e != cudaSuccess) {
        cudaFree(t->q);
        cudaFree(t->d);
        cudaFree(t->status);
        return cuda_err(e, "tensor status word");
    }
    if (qb::gemm_tc_supported(t->m)) {
        e = cudaMalloc(&t->tcbuf, qb::tc_weight_bytes(t->m));
        if (e == cudaSuccess) e = qb::tc_prepare_weights(t->m, t->tcbuf, &t->wmap, nullptr);
        if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
        if (e != cudaSuccess) {
            cudaFree(t->q);
            cudaFree(t->d);
            cudaFree(t->status);
            cudaFree(t->tcbuf);
            return cuda_err(e, "tensor-core weight copies");
        }
        t->tc = true;
    }
    *out = t.release();
    return QNT_OK;
}

int qnt_tensor_free(qnt_dtensor* t) {
    if (!t) return QNT_OK;
    cudaFree(t->q);
    cudaFree(t->d);
    cudaFree(t->status);
    cudaFree(t->tcbuf);
    delete t;
    return QNT_OK;
}

int qnt_tensor_shape(const qnt_dtensor* t, int* dtype, int* rows, int* cols) {
    if (!t) return set_err(QNT_ERR_INVALID, "null tensor");
    if (dtype) *dtype = t->m.dtype;
    if (rows) *rows = t->m.rows;
    if (cols) *cols = t->m.cols;
    return QNT_OK;
}

int qnt_quantize_q8(const float* x, int n_tok, int n, int8_t* q, float* d, void* stream) {
    if (n_tok < 0 || n < 0 || n % 32) return set_err(QNT_ERR_INVALID, "n must be a multiple of 32");
    cudaError_t e = qb::launch_quantize_q8(x, n_tok, n, q, d, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? QNT_OK : cuda_err(e, "quantize_q8");
}

int qnt_matvec(const qnt_dtensor* W, const int8_t* qx, const float* dx, int r0, int r1, float* out, void* stream) {
    if (!W || r0 < 0 || r1 > W->m.rows || r0 > r1) return set_err(QNT_ERR_INVALID, "bad row range");
    if (W->m.cols > 16384) return set_err(QNT_ERR_UNSUPPORTED, "matvec supports cols <= 16384");
    cudaError_t e = qb::launch_matvec(W->m, qx, dx, r0, r1, out, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? QNT_OK : cuda_err(e, "matvec");
}

int qnt_matmul(const qnt_dtensor* W, const int8_t* qx, const float* dx, int n, int r0, int r1, float* out, int ldo, int impl,
               void* stream) {
    if (!W || r0 < 0 || r1 > W->m.rows || r0 > r1 || n < 0 || ldo < r1) return set_err(QNT_ERR_INVALID, "bad matmul arguments");
    if (impl < 0 || impl > 2) return set_err(QNT_ERR_INVALID, "impl must be 0 (auto), 1 (CUDA cores) or 2 (tensor cores)");
    const bool tc = impl == 2 || (impl == 0 && W->tc && n >= qb::kTcMinTokens);
    cudaError_t e;
    if (tc) {
        if (!W->tc) return set_err(QNT_ERR_UNSUPPORTED, "tensor-core matmul needs cols % 128 == 0 and a TMA-capable driver");
        if ((reinterpret_cast<uintptr_t>(qx) | reinterpret_cast<uintptr_t>(dx)) & 15)
            return set_err(QNT_ERR_INVALID, "tensor-core matmul needs 16-byte aligned activations");
        if (n == 0 || r1 == r0) return QNT_OK;
        // the kernel reads the activation scales block-major: a stream-ordered transposed copy
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        const int nb = W->m.cols / 32, ldt = (n + 31) & ~31;
        float* dxt = nullptr;
        e = cudaMallocAsync(reinterpret_cast<void**>(&dxt), size_t(nb) * ldt * 4, s);
        if (e != cudaSuccess) return cuda_err(e, "matmul scale copy");
        qb::TcAct act;
        e = qb::launch_transpose_scales(dx, n, nb, dxt, ldt, s);
        if (e == cudaSuccess && !qb::make_act_maps(qx, dxt, n, ldt, W->m.cols, &act)) e = cudaErrorInvalidValue;
        if (e == cudaSuccess) e = qb::launch_matmul_tc(W->m, W->wmap, act, n, r0, r1, out, ldo, W->status, s);
        const cudaError_t ef = cudaFreeAsync(dxt, s);
        if (e == cudaSuccess) e = ef;
    } else {
        e = qb::launch_matmul_simt(W->m, qx, dx, n, r0, r1, out, ldo, static_cast<cudaStream_t>(stream));
    }
    return e == cudaSuccess ? QNT_OK : cuda_err(e, "matmul");
}

int qnt_quantize_q8_host(const float* x, int n, int8_t* q, float* d) {
    if (n <= 0 || n % 32) return set_err(QNT_ERR_INVALID, "n must be a positive multiple of 32");
    float* dxv = nullptr;
    int8_t* dq = nullptr;
    float* dd = nullptr;
    cudaError_t e = cudaMalloc(&dxv, size_t(n) * 4);
    if (e == cudaSuccess) e = cudaMalloc(&dq, size_t(n));
    if (e == cudaSuccess) e = cudaMalloc(&dd, size_t(n / 32) * 4);
    if (e == cudaSuccess) e = cudaMemcpy(dxv, x, size_t(n) * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = qb::launch_quantize_q8(dxv, 1, n, dq, dd, nullptr);
    if (e == cudaSuccess) e = cudaMemcpy(q, dq, size_t(n), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(d, dd, size_t(n / 32) * 4, cudaMemcpyDeviceToHost);
    cudaFree(dxv);
    cudaFree(dq);
    cudaFree(dd);
    return e == cudaSuccess ? QNT_OK : cuda_err(e, "quantize_q8_host");
}

static int host_mm(const qnt_dtensor* W, const int8_t* qx, const float* dx, int n, int r0, int r1, float* out, int ldo, bool mv,
                   int impl) {
    if (!W || r0 < 0 || r1 > W->m.rows || r0 > r1 || n <= 0) return set_err(QNT_ERR_INVALID, "bad arguments");
    const int cols = W->m.cols;
    int8_t* dq = nullptr;
    float *dd = nullptr, *dout = nullptr;
    const size_t out_elems = mv ? size_t(r1) : size_t(n - 1) * ldo + r1;
    cudaError_t e = cudaMalloc(&dq, size_t(n) * cols);
    if (e == cudaSuccess) e = cudaMalloc(&dd, size_t(n) * (cols / 32) * 4);
    if (e == cudaSuccess) e = cudaMalloc(&dout, out_elems * 4);
    if (e == cudaSuccess) e = cudaMemcpy(dq, qx, size_t(n) * cols, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(dd, dx, size_t(n) * (cols / 32) * 4, cudaMemcpyHostToDevice);
    int rc = QNT_OK;
    if (e == cudaSuccess) {
        rc = mv ? qnt_matvec(W, dq, dd, r0, r1, dout, nullptr) : qnt_matmul(W, dq, dd, n, r0, r1, dout, ldo, impl, nullptr);
        e = cudaDeviceSynchronize();
    }
    if (e == cudaSuccess && rc == QNT_OK) {
        unsigned st = 0;
        e = cudaMemcpy(&st, W->status, sizeof st, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && st) {
            cudaMemset(W->status, 0, sizeof st);
            rc = set_err(QNT_ERR_DEVICE, "matmul kernel reported status bits " + std::to_string(st));
        }
    }
    if (e == cudaSuccess && rc == QNT_OK) {
        if (mv) {
            e = cudaMemcpy(out + r0, dout + r0, size_t(r1 - r0) * 4, cudaMemcpyDeviceToHost);
        } else {
            for (int t = 0; t < n && e == cudaSuccess; ++t)
                e = cudaMemcpy(out + size_t(t) * ldo + r0, dout + size_t(t) * ldo + r0, size_t(r1 - r0) * 4,
                               cudaMemcpyDeviceToHost);
        }
    }
    cudaFree(dq);
    cudaFree(dd);
    cudaFree(dout);
    if (rc != QNT_OK) return rc;
    return e == cudaSuccess ? QNT_OK : cuda_err(e, "host matvec/matmul");
}

int qnt_matvec_host(const qnt_dtensor* W, const int8_t* qx, const float* dx, int r0, int r1, float* out) {
    return host_mm(W, qx, dx, 1, r0, r1, out, 0, true, 0);
}

int qnt_matmul_host(const qnt_dtensor* W, const int8_t* qx, const float* dx, int n, int r0, int r1, float* out, int ldo,
                    int impl) {
    if (ldo < r1) return set_err(QNT_ERR_INVALID, "ldo < r1");
    return host_mm(W, qx, dx, n, r0, r1, out, ldo, false, impl);
}

// ---------------------------------------------------------------- model level

int qnt_model_open(const char* path, int ctx_len, int flags, qnt_model** out) {
    (void)flags;
    if (!path || !out) return set_err(QNT_ERR_INVALID, "null argument");
    auto m = std::make_unique<qnt_model>();
    std::string err;
    if (!m->eng.load(path, ctx_len, &err)) return set_err(m->eng.file_fault() ? QNT_ERR_IO : QNT_ERR_UNSUPPORTED, err);
    *out = m.release();
    return QNT_OK;
}

void qnt_model_close(qnt_model* m) { delete m; }

int qnt_model_hparams(const qnt_model* m, qnt_hparams* out) {
    if (!m || !out) return set_err(QNT_ERR_INVALID, "null argument");
    const qb::HParams& h = m->eng.hparams();
    out->vocab_size = h.vocab_size;
    out->dim = h.dim;
    out->n_layers = h.n_layers;
    out->n_heads = h.n_heads;
    out->n_kv_heads = h.n_kv_heads;
    out->head_dim = h.head_dim;
    out->ffn_dim = h.ffn_dim;
    out->max_seq = h.max_seq;
    out->rope_theta = h.rope_theta;
    out->norm_eps = h.norm_eps;
    out->tied_embeddings = h.tied_embeddings;
    out->qkv_bias = h.qkv_bias;
    out->flags = h.flags;
    out->n_tokens = m->eng.n_valid_default();
    out->ctx_len = m->eng.ctx_len();
    out->has_shortlist = m->eng.has_shortlist() ? 1 : 0;
    return QNT_OK;
}

static qb::HeadQueryC to_hq(const qnt_head_query* hq) {
    qb::HeadQueryC q;
    if (hq) {
        q.top_k = hq->top_k;
        q.n_valid = hq->n_valid;
        q.must = hq->must;
        q.n_must = hq->n_must;
    }
    return q;
}

int qnt_model_forward(qnt_model* m, int token, int pos, const qnt_head_query* hq, float* logits) {
    if (!m) return set_err(QNT_ERR_INVALID, "null model");
    const qb::HeadQueryC q = to_hq(hq);
    return engine_code(m->eng, m->eng.forward(token, pos, hq ? &q : nullptr, logits));
}

int qnt_model_forward_batch(qnt_model* m, const int* tokens, int n, int pos0, const qnt_head_query* hq, float* logits) {
    if (!m || !tokens) return set_err(QNT_ERR_INVALID, "null argument");
    const qb::HeadQueryC q = to_hq(hq);
    return engine_code(m->eng, m->eng.forward_batch(tokens, n, pos0, hq ? &q : nullptr, logits));
}

int qnt_model_head(qnt_model* m, const qnt_head_query* hq, float* logits, float* coarse, float* upper) {
    if (!m) return set_err(QNT_ERR_INVALID, "null model");
    const qb::HeadQueryC q = to_hq(hq);
    return engine_code(m->eng, m->eng.head(hq ? &q : nullptr, logits, coarse, upper));
}

int qnt_model_last_head_rows(const qnt_model* m) { return m ? m->eng.last_head_rows() : 0; }
int qnt_model_has_shortlist(const qnt_model* m) { return m && m->eng.has_shortlist() ? 1 : 0; }
size_t qnt_model_kv_cache_bytes(const qnt_model* m) { return m ? m->eng.kv_cache_bytes() : 0; }
size_t qnt_model_weight_bytes(const qnt_model* m) { return m ? m->eng.weight_bytes() : 0; }

int qnt_generate(qnt_model* m, const int* prompt, int n_prompt, const qnt_sampler_params* sp, int flags, int n_gen,
                 int* out_ids, qnt_gen_stats* stats) {
    if (!m || !prompt || !sp || (n_gen > 0 && !out_ids)) return set_err(QNT_ERR_INVALID, "null argument");
    qb::SamplerParamsC p;
    p.temperature = sp->temperature;
    p.top_k = sp->top_k;
    p.top_p = sp->top_p;
    p.min_p = sp->min_p;
    p.repeat_penalty = sp->repeat_penalty;
    p.repeat_window = sp->repeat_window;
    p.seed = sp->seed;
    qb::GenStats gs;
    const int r = m->eng.generate(prompt, n_prompt, p, (flags & QNT_GEN_SHORTLIST) != 0, (flags & QNT_GEN_BATCH_PREFILL) != 0,
                                  n_gen, out_ids, &gs);
    if (r < 0) return engine_code(m->eng, r);
    if (stats) {
        stats->prefill_ms = gs.prefill_ms;
        stats->decode_ms = gs.decode_ms;
        stats->head_rows = gs.head_rows;
        stats->head_calls = gs.head_calls;
        stats->kernels_per_step = m->eng.kernels_per_step();
    }
    return r;
}

int qnt_session_begin(qnt_model* m, const int* prompt, int n_prompt, const qnt_sampler_params* sp, int flags) {
    if (!m || !prompt || !sp) return set_err(QNT_ERR_INVALID, "null argument");
    qb::SamplerParamsC p;
    p.temperature = sp->temperature;
    p.top_k = sp->top_k;
    p.top_p = sp->top_p;
    p.min_p = sp->min_p;
    p.repeat_penalty = sp->repeat_penalty;
    p.repeat_window = sp->repeat_window;
    p.seed = sp->seed;
    return engine_code(m->eng, m->eng.session_begin(prompt, n_prompt, p, (flags & QNT_GEN_SHORTLIST) != 0,
                                                    (flags & QNT_GEN_BATCH_PREFILL) != 0));
}

int qnt_session_step(qnt_model* m, int n) {
    if (!m || n < 0) return set_err(QNT_ERR_INVALID, "bad argument");
    return engine_code(m->eng, m->eng.session_step(n));
}

int qnt_session_read(qnt_model* m, int* out_ids, int max_ids, qnt_gen_stats* stats) {
    if (!m || (max_ids > 0 && !out_ids)) return set_err(QNT_ERR_INVALID, "null argument");
    qb::GenStats gs;
    const int r = m->eng.session_read(out_ids, max_ids, &gs);
    if (r < 0) return engine_code(m->eng, r);
    if (stats) {
        stats->prefill_ms = 0;
        stats->decode_ms = 0;
        stats->head_rows = gs.head_rows;
        stats->head_calls = gs.head_calls;
        stats->kernels_per_step = m->eng.kernels_per_step();
    }
    return r;
}

int qnt_batch_init(qnt_model* m, int max_seqs, int ctx_len) {
    if (!m) return set_err(QNT_ERR_INVALID, "null model");
    return engine_code(m->eng, m->eng.batch_init(max_seqs, ctx_len));
}

int qnt_prefill_batch(qnt_model* m, int seq, const int* tokens, int n, int* next_id) {
    if (!m) return set_err(QNT_ERR_INVALID, "null model");
    return engine_code(m->eng, m->eng.batch_prefill(seq, tokens, n, next_id));
}

int qnt_decode_batch(qnt_model* m, const int* seq_ids, const int* tokens, int n, int* next_ids) {
    if (!m) return set_err(QNT_ERR_INVALID, "null model");
    return engine_code(m->eng, m->eng.batch_decode(seq_ids, tokens, n, next_ids));
}

int qnt_batch_reset(qnt_model* m, int seq) {
    if (!m) return set_err(QNT_ERR_INVALID, "null model");
    return engine_code(m->eng, m->eng.batch_reset(seq));
}

int qnt_model_debug_buffer(qnt_model* m, int what, float* out) {
    if (!m || !out) return set_err(QNT_ERR_INVALID, "null argument");
    return m->eng.debug_buffer(what, out);
}

void* qnt_model_stream(const qnt_model* m) { return m ? static_cast<void*>(m->eng.stream()) : nullptr; }

}  // extern "C"
