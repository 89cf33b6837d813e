// extern "C" layer of include/quanta_b200.h over the engine and the ops-level kernels.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "quanta_b200.h"
#include "capi_util.h"
#include "engine.h"
#include "gemm_tc.h"
#include "ops.h"
#include "tokenizer.h"

struct qnt_dtensor {
    qb::DMat m;
    void* q = nullptr;
    void* d = nullptr;
    qb::TcMap wmap{};          // TMA source for the tensor-core matmul
    bool tc = false;           // wmap is valid
    void* tcbuf = nullptr;     // the copies wmap reads (stage-major scales; Q4_0: int8 q - 8)
};

struct qnt_model {
    qb::Engine eng;
};

struct qnt_tokenizer {
    qb::QntFile file;
    std::unique_ptr<qb::BpeTokenizer> bpe;
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

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// What each calling thread keeps for the ops-level entries, per device: a status word of its own (the tensor-core
// matmul's bounded waits report there, so concurrent callers never see or clear each other's bits), and for the
// synchronous host entries one stream with device and pinned host staging that only grows -- a call allocates
// nothing once its sizes have been seen, and synchronises only its own stream.
struct ThreadOps {
    int device = -1;
    cudaStream_t st = nullptr;
    unsigned* status = nullptr;     // device word
    unsigned* status_h = nullptr;   // pinned copy read after a host call
    unsigned char* dbuf = nullptr;  // device staging
    size_t dcap = 0;
    unsigned char* hbuf = nullptr;  // pinned host staging
    size_t hcap = 0;

    ~ThreadOps() { release(); }
    void release() {
        if (device < 0) return;
        int cur = -1;
        cudaGetDevice(&cur);
        cudaSetDevice(device);
        if (st) cudaStreamDestroy(st);
        cudaFree(status);
        cudaFree(dbuf);
        cudaFreeHost(status_h);
        cudaFreeHost(hbuf);
        if (cur >= 0) cudaSetDevice(cur);
        *this = ThreadOps{};
        device = -1;
    }
    // the current device's stream and status word (made on first use)
    cudaError_t ready() {
        int dev = -1;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev == device) return cudaSuccess;
        release();
        device = dev;
        e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaMalloc(&status, sizeof(unsigned));
        if (e == cudaSuccess) e = cudaMemset(status, 0, sizeof(unsigned));
        if (e == cudaSuccess) e = cudaMallocHost(&status_h, sizeof(unsigned));
        if (e != cudaSuccess) release();
        return e;
    }
    cudaError_t staging(size_t dbytes, size_t hbytes) {
        cudaError_t e = ready();
        if (e == cudaSuccess && dbytes > dcap) {
            cudaFree(dbuf);
            dbuf = nullptr;
            dcap = 0;
            e = cudaMalloc(&dbuf, dbytes);
            if (e == cudaSuccess) dcap = dbytes;
        }
        if (e == cudaSuccess && hbytes > hcap) {
            cudaFreeHost(hbuf);
            hbuf = nullptr;
            hcap = 0;
            e = cudaMallocHost(&hbuf, hbytes);
            if (e == cudaSuccess) hcap = hbytes;
        }
        return e;
    }
};

thread_local ThreadOps t_ops;

// The tensor-core or CUDA-core matmul on device pointers.  dxt: a block-major scale buffer of nb * ((n + 31) & ~31)
// floats, or null to take one stream-ordered from the pool for this call.
int matmul_dev(const qnt_dtensor* W, const int8_t* qx, const float* dx, int n, int r0, int r1, float* out, int ldo, int impl,
               cudaStream_t s, unsigned* status, float* dxt) {
    const bool tc = impl == 2 || (impl == 0 && W->tc && n >= qb::kTcMinTokens);
    cudaError_t e;
    if (tc) {
        if (!W->tc) return set_err(QNT_ERR_UNSUPPORTED, "tensor-core matmul needs cols % 128 == 0 and a TMA-capable driver");
        if ((reinterpret_cast<uintptr_t>(qx) | reinterpret_cast<uintptr_t>(dx)) & 15)
            return set_err(QNT_ERR_INVALID, "tensor-core matmul needs 16-byte aligned activations");
        if (n == 0 || r1 == r0) return QNT_OK;
        // the kernel reads the activation scales block-major: a stream-ordered transposed copy
        const int nb = W->m.cols / 32, ldt = (n + 63) & ~63;  // a whole number of the kernel's 64-token tiles
        const bool own = dxt == nullptr;
        if (own) {
            e = cudaMallocAsync(reinterpret_cast<void**>(&dxt), size_t(nb) * ldt * 4, s);
            if (e != cudaSuccess) return cuda_err(e, "matmul scale copy");
        }
        qb::TcAct act;
        e = qb::launch_transpose_scales(dx, n, nb, dxt, ldt, s);
        if (e == cudaSuccess && !qb::make_act_maps(qx, dxt, n, ldt, W->m.cols, &act)) e = cudaErrorInvalidValue;
        if (e == cudaSuccess) e = qb::launch_matmul_tc(W->m, W->wmap, act, n, r0, r1, out, ldo, status, s);
        if (own) {
            const cudaError_t ef = cudaFreeAsync(dxt, s);
            if (e == cudaSuccess) e = ef;
        }
    } else {
        e = qb::launch_matmul_simt(W->m, qx, dx, n, r0, r1, out, ldo, s);
    }
    return e == cudaSuccess ? QNT_OK : cuda_err(e, "matmul");
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
    if (qb::gemm_tc_supported(t->m)) {
        e = cudaMalloc(&t->tcbuf, qb::tc_weight_bytes(t->m));
        if (e == cudaSuccess) e = qb::tc_prepare_weights(t->m, t->tcbuf, &t->wmap, nullptr);
        if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
        if (e != cudaSuccess) {
            cudaFree(t->q);
            cudaFree(t->d);
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
    const cudaError_t e = t_ops.ready();
    if (e != cudaSuccess) return cuda_err(e, "matmul set-up");
    return matmul_dev(W, qx, dx, n, r0, r1, out, ldo, impl, static_cast<cudaStream_t>(stream), t_ops.status, nullptr);
}

int qnt_ops_check(void* stream) {
    cudaError_t e = t_ops.ready();
    if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    unsigned st = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&st, t_ops.status, sizeof st, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && st) e = cudaMemset(t_ops.status, 0, sizeof st);
    if (e != cudaSuccess) return cuda_err(e, "qnt_ops_check");
    if (st) return set_err(QNT_ERR_DEVICE, "an ops-level kernel of this thread reported status bits " + std::to_string(st));
    return QNT_OK;
}

int qnt_quantize_q8_host(const float* x, int n, int8_t* q, float* d) {
    if (n <= 0 || n % 32 || !x || !q || !d) return set_err(QNT_ERR_INVALID, "n must be a positive multiple of 32");
    const size_t xb = size_t(n) * 4, qb_ = align256(size_t(n)), db = size_t(n / 32) * 4;
    const size_t qoff = align256(xb), doff = qoff + qb_, total = doff + db;
    cudaError_t e = t_ops.staging(total, total);
    if (e != cudaSuccess) return cuda_err(e, "quantize_q8_host staging");
    std::memcpy(t_ops.hbuf, x, xb);
    e = cudaMemcpyAsync(t_ops.dbuf, t_ops.hbuf, xb, cudaMemcpyHostToDevice, t_ops.st);
    if (e == cudaSuccess)
        e = qb::launch_quantize_q8(reinterpret_cast<const float*>(t_ops.dbuf), 1, n, reinterpret_cast<int8_t*>(t_ops.dbuf + qoff),
                                   reinterpret_cast<float*>(t_ops.dbuf + doff), t_ops.st);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(t_ops.hbuf + qoff, t_ops.dbuf + qoff, total - qoff, cudaMemcpyDeviceToHost, t_ops.st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(t_ops.st);
    if (e != cudaSuccess) return cuda_err(e, "quantize_q8_host");
    std::memcpy(q, t_ops.hbuf + qoff, size_t(n));
    std::memcpy(d, t_ops.hbuf + doff, db);
    return QNT_OK;
}

// The synchronous host entries: inputs through pinned staging to the thread's device staging, the kernel on the
// thread's stream, the used output rows back, and the thread's status word checked.  Device layout:
// [q n x cols | d n x nb | block-major d nb x ldt | out n x r1].
static int host_mm(const qnt_dtensor* W, const int8_t* qx, const float* dx, int n, int r0, int r1, float* out, int ldo, bool mv,
                   int impl) {
    if (!W || !qx || !dx || !out || r0 < 0 || r1 > W->m.rows || r0 > r1 || n <= 0)
        return set_err(QNT_ERR_INVALID, "bad arguments");
    if (r0 == r1) return QNT_OK;
    const int cols = W->m.cols, nb = cols / 32, ldt = (n + 63) & ~63;
    const size_t qbytes = size_t(n) * cols, dbytes = size_t(n) * nb * 4;
    const size_t doff = align256(qbytes), toff = doff + align256(dbytes), ooff = toff + align256(size_t(nb) * ldt * 4);
    const size_t obytes = size_t(n) * r1 * 4;
    // host staging: [q | d | out], with the out block at the same offset as on the device
    cudaError_t e = t_ops.staging(ooff + obytes, ooff + obytes);
    if (e != cudaSuccess) return cuda_err(e, "host matvec/matmul staging");
    unsigned char* h = t_ops.hbuf;
    unsigned char* dv = t_ops.dbuf;
    std::memcpy(h, qx, qbytes);
    std::memcpy(h + doff, dx, dbytes);
    e = cudaMemcpyAsync(dv, h, doff + dbytes, cudaMemcpyHostToDevice, t_ops.st);
    if (e != cudaSuccess) return cuda_err(e, "host matvec/matmul input copy");
    const int8_t* dq = reinterpret_cast<const int8_t*>(dv);
    const float* dd = reinterpret_cast<const float*>(dv + doff);
    float* dout = reinterpret_cast<float*>(dv + ooff);
    int rc;
    if (mv) {
        if (cols > 16384) return set_err(QNT_ERR_UNSUPPORTED, "matvec supports cols <= 16384");
        e = qb::launch_matvec(W->m, dq, dd, r0, r1, dout, t_ops.st);
        rc = e == cudaSuccess ? QNT_OK : cuda_err(e, "matvec");
    } else {
        rc = matmul_dev(W, dq, dd, n, r0, r1, dout, r1, impl, t_ops.st, t_ops.status, reinterpret_cast<float*>(dv + toff));
    }
    if (rc != QNT_OK) return rc;
    e = cudaMemcpyAsync(h + ooff, dout, obytes, cudaMemcpyDeviceToHost, t_ops.st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(t_ops.status_h, t_ops.status, sizeof(unsigned), cudaMemcpyDeviceToHost, t_ops.st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(t_ops.st);
    if (e != cudaSuccess) return cuda_err(e, "host matvec/matmul");
    if (const unsigned st = *t_ops.status_h) {
        cudaMemsetAsync(t_ops.status, 0, sizeof(unsigned), t_ops.st);
        cudaStreamSynchronize(t_ops.st);
        return set_err(QNT_ERR_DEVICE, "matmul kernel reported status bits " + std::to_string(st));
    }
    const float* ho = reinterpret_cast<const float*>(h + ooff);
    for (int t = 0; t < (mv ? 1 : n); ++t)
        std::memcpy(out + size_t(t) * ldo + r0, ho + size_t(t) * r1 + r0, size_t(r1 - r0) * 4);
    return QNT_OK;
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
    if (!path || !out) return set_err(QNT_ERR_INVALID, "null argument");
    if (flags & ~QNT_OPEN_NIBBLE_SCREEN) return set_err(QNT_ERR_INVALID, "unknown qnt_model_open flags");
    auto m = std::make_unique<qnt_model>();
    std::string err;
    if (!m->eng.load(path, ctx_len, &err, (flags & QNT_OPEN_NIBBLE_SCREEN) != 0)) return set_err(m->eng.file_fault() ? QNT_ERR_IO : QNT_ERR_UNSUPPORTED, err);
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

int qnt_export_device_layout(const char* in_path, const char* out_path) {
    if (!in_path || !out_path) return set_err(QNT_ERR_INVALID, "null argument");
    std::string err;
    if (!qb::export_device_layout(in_path, out_path, &err)) return set_err(QNT_ERR_IO, err);
    return QNT_OK;
}

int qnt_model_packed_tensors(const qnt_model* m) { return m ? m->eng.packed_tensors() : 0; }

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
                                                    (flags & QNT_GEN_BATCH_PREFILL) != 0, (flags & QNT_GEN_KEEP_RNG) != 0));
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

int qnt_model_nll(qnt_model* m, const int* ids, int n, double* nll) {
    if (!m || !nll || n < 0 || (n > 0 && !ids)) return set_err(QNT_ERR_INVALID, "bad argument");
    return engine_code(m->eng, m->eng.nll(ids, n, nll));
}

int qnt_session_feed(qnt_model* m, const int* ids, int n) {
    if (!m || (n > 0 && !ids) || n < 0) return set_err(QNT_ERR_INVALID, "bad argument");
    return engine_code(m->eng, m->eng.session_feed(ids, n));
}

int qnt_session_rewind(qnt_model* m, int n_drop) {
    if (!m) return set_err(QNT_ERR_INVALID, "null model");
    return engine_code(m->eng, m->eng.session_rewind(n_drop));
}

int qnt_session_last(qnt_model* m, int* token, int* length) {
    if (!m) return set_err(QNT_ERR_INVALID, "null model");
    return engine_code(m->eng, m->eng.session_last(token, length));
}

// ---------------------------------------------------------------- text

int qnt_tokenizer_open(const char* path, qnt_tokenizer** out) {
    if (!path || !out) return set_err(QNT_ERR_INVALID, "null argument");
    *out = nullptr;
    auto t = std::make_unique<qnt_tokenizer>();
    std::string err;
    if (!t->file.open(path, &err)) return set_err(QNT_ERR_IO, err);
    try {
        t->bpe = std::make_unique<qb::BpeTokenizer>(t->file.tokenizer());
    } catch (const std::exception& e) {
        return set_err(QNT_ERR_IO, e.what());
    }
    *out = t.release();
    return QNT_OK;
}

void qnt_tokenizer_free(qnt_tokenizer* t) { delete t; }

int qnt_tokenizer_n_tokens(const qnt_tokenizer* t) { return t ? t->bpe->n_tokens() : 0; }

int qnt_tokenize(const qnt_tokenizer* t, const char* text, size_t len, int* ids, int max_ids) {
    if (!t || (len > 0 && !text) || max_ids < 0 || (max_ids > 0 && !ids)) return set_err(QNT_ERR_INVALID, "bad argument");
    const std::vector<int> v = t->bpe->encode(std::string(text ? text : "", len));
    if (v.size() > size_t(INT32_MAX)) return set_err(QNT_ERR_RANGE, "text encodes to too many tokens");
    std::memcpy(ids, v.data(), std::min(v.size(), size_t(max_ids)) * sizeof(int));
    return int(v.size());
}

int qnt_token_piece(const qnt_tokenizer* t, int id, char* buf, int cap) {
    if (!t || cap < 0 || (cap > 0 && !buf)) return set_err(QNT_ERR_INVALID, "bad argument");
    const std::string& p = t->bpe->piece(id);
    std::memcpy(buf, p.data(), std::min(p.size(), size_t(cap)));
    return int(p.size());
}

int qnt_token_id(const qnt_tokenizer* t, const char* literal) {
    if (!t || !literal) return -1;
    return t->bpe->special_id(literal);
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

int qnt_wait_probe(unsigned limit, void* stream) {
    if (limit == 0 || limit > (1u << 20)) return set_err(QNT_ERR_INVALID, "qnt_wait_probe: 0 < limit <= 2^20 tries");
    cudaError_t e = t_ops.ready();
    if (e == cudaSuccess) e = qb::launch_wait_probe(limit, t_ops.status, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_err(e, "qnt_wait_probe");
    return qnt_ops_check(stream);
}

int qnt_bench_mma_i8(int iters, double* tops) {
    if (iters <= 0 || !tops) return set_err(QNT_ERR_INVALID, "qnt_bench_mma_i8: iters > 0 and an output needed");
    unsigned status = 0;
    const cudaError_t e = qb::bench_mma_i8(iters, tops, &status);
    if (e != cudaSuccess) return cuda_err(e, "qnt_bench_mma_i8");
    if (status) return set_err(QNT_ERR_DEVICE, "qnt_bench_mma_i8: the MMA completion wait timed out");
    return QNT_OK;
}

}  // extern "C"
