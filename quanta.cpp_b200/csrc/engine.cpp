#include "engine.h"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <stdexcept>

namespace qb {

namespace {

size_t align_up(size_t n, size_t a) { return (n + a - 1) / a * a; }

}  // namespace

Engine::~Engine() {
    if (st_) cudaStreamSynchronize(st_);
    for (auto& g : graphs_) cudaGraphExecDestroy(g.second);
    for (void* p : allocs_) cudaFree(p);
    cudaFree(bkcache_);
    cudaFree(bvcache_);
    if (st_) cudaStreamDestroy(st_);
}

bool Engine::fail(const std::string& m) {
    err_ = m;
    return false;
}

int Engine::cuda_fail(cudaError_t e, const char* what) {
    err_ = std::string(what) + ": " + cudaGetErrorString(e);
    return -2;
}

void* Engine::dalloc(size_t bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, align_up(std::max<size_t>(bytes, 1), 256)) != cudaSuccess) throw std::runtime_error("cudaMalloc failed");
    allocs_.push_back(p);
    return p;
}

bool Engine::tc_weights(const DMat& W, TcMap* map) {
    if (!gemm_tc_supported(W)) return false;
    const size_t b = tc_weight_bytes(W);
    void* buf = dalloc(b);
    tc_copy_bytes_ += b;
    return tc_prepare_weights(W, buf, map, st_) == cudaSuccess;
}

int Engine::n_valid_default() const {
    return std::min(file_.tokenizer().n_tokens > 0 ? file_.tokenizer().n_tokens : hp_.vocab_size, hp_.vocab_size);
}

// Quantized matrix: quants then fp16 scales, each in its own 256-byte aligned device array.
DMat Engine::upload_matrix(const HostTensor& t) {
    if (t.dtype != DT_Q8_0 && t.dtype != DT_Q4_0)
        throw std::runtime_error("weight matrices must be q8_0 or q4_0 on the device");
    DMat m;
    m.dtype = t.dtype;
    m.rows = t.rows;
    m.cols = t.cols;
    const size_t qb = t.quant_bytes(), sb = size_t(t.rows) * (t.cols / QK) * 2;
    void* q = dalloc(qb);
    void* d = dalloc(sb);
    if (cudaMemcpy(q, t.data, qb, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(d, t.data + qb, sb, cudaMemcpyHostToDevice) != cudaSuccess)
        throw std::runtime_error("upload failed");
    m.q = static_cast<const uint8_t*>(q);
    m.d = static_cast<const __half*>(d);
    weight_bytes_ += qb + sb;
    return m;
}

// Fused matrices in the device's row order (fuse_rows, device_layout.h).  mode 0: q|k|v, rows pair-interleaved per
// head (row i and i + head_dim/2 adjacent); mode 1: gate|up interleaved per 32 rows (64j..64j+31 gate block j,
// 64j+32..64j+63 up block j).
DMat Engine::upload_fused(const std::vector<const HostTensor*>& parts, int mode) {
    const FusedHost f = fuse_rows(parts, mode, hp_.head_dim);
    DMat m;
    m.dtype = f.dtype;
    m.rows = f.rows;
    m.cols = f.cols;
    void* q = dalloc(f.q.size());
    void* d = dalloc(f.d.size() * 2);
    if (cudaMemcpy(q, f.q.data(), f.q.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(d, f.d.data(), f.d.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess)
        throw std::runtime_error("upload failed");
    m.q = static_cast<const uint8_t*>(q);
    m.d = static_cast<const __half*>(d);
    weight_bytes_ += f.q.size() + f.d.size() * 2;
    return m;
}

// A fused matrix stored pre-packed by export_device_layout: uploaded as it is when it holds the parts' rows in the
// fused order (dtype, shape and a sample of rows checked), else fused here.
DMat Engine::upload_packed(const HostTensor* packed, const std::vector<const HostTensor*>& parts, int mode) {
    if (packed && packed_rows_match(*packed, parts, mode, hp_.head_dim)) {
        ++packed_tensors_;
        return upload_matrix(*packed);
    }
    return upload_fused(parts, mode);
}

bool Engine::load(const std::string& path, int ctx_len, std::string* err, bool nibble_screen) {
    auto bad = [&](const std::string& m) {
        err_ = m;
        if (err) *err = m;
        return false;
    };
    std::string e;
    file_fault_ = false;
    if (!file_.open(path, &e)) {
        file_fault_ = true;
        return bad(e);
    }
    hp_ = file_.hparams();
    if (hp_.n_heads * hp_.head_dim != hp_.dim || hp_.n_kv_heads <= 0 || hp_.n_heads % hp_.n_kv_heads != 0)
        return bad("unsupported head configuration");
    if (hp_.head_dim != 64) return bad("the device attention kernel needs head_dim == 64");
    if (hp_.n_heads / hp_.n_kv_heads > 8) return bad("the device attention kernel needs <= 8 query heads per kv head");
    if (hp_.dim % QK || hp_.ffn_dim % QK || hp_.dim > 8192 || hp_.ffn_dim > 16384) return bad("unsupported dims");
    // FLAG_HADAMARD_DOWN (block-256 transform of the SwiGLU output before down), validated as model.cpp:39 does
    hadamard_ = (hp_.flags & 1u) != 0;
    if (hadamard_ && hp_.ffn_dim % 256 != 0) return bad("FLAG_HADAMARD_DOWN needs ffn_dim % 256 == 0");
    ctx_ = (ctx_len > 0 && ctx_len < hp_.max_seq) ? ctx_len : hp_.max_seq;
    if (cudaGetDevice(&device_) != cudaSuccess) return bad("no CUDA device");
    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, device_);
    if (prop.major < 10) return bad("this build needs an sm_100 (Blackwell) GPU");
    n_sm_ = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking) != cudaSuccess) return bad("stream create failed");
    // Launch-mode switches for diagnosis (defaults: programmatic dependent launch on, CUDA graphs on).
    if (const char* v = std::getenv("QNT_PDL")) pdl_ = std::atoi(v) != 0;
    if (const char* v = std::getenv("QNT_GRAPHS")) use_graphs_ = std::atoi(v) != 0;
    if (const char* v = std::getenv("QNT_FUSE_QKV")) fuse_qkv_attn_ = std::atoi(v) != 0;
    if (const char* v = std::getenv("QNT_FUSE_O")) fuse_o_ = std::atoi(v) != 0;
    if (const char* v = std::getenv("QNT_TC_SWIGLU")) tc_swiglu_ = std::atoi(v) != 0;
    if (const char* v = std::getenv("QNT_TC_QKV")) tc_qkv_ = std::atoi(v) != 0;
    try {
        const HostTensor& emb = file_.require("model.embed_tokens.weight");
        embed_ = upload_matrix(emb);
        lm_head_ = hp_.tied_embeddings ? embed_ : upload_matrix(file_.require("lm_head.weight"));
        const HostTensor& fn = file_.require("model.norm.weight");
        auto upload_f32 = [&](const HostTensor& t) {
            if (t.dtype != DT_F32) throw std::runtime_error("norms and biases must be f32");
            void* p = dalloc(size_t(t.cols) * t.rows * 4);
            cudaMemcpy(p, t.data, size_t(t.cols) * t.rows * 4, cudaMemcpyHostToDevice);
            weight_bytes_ += size_t(t.cols) * t.rows * 4;
            return static_cast<const float*>(p);
        };
        final_norm_ = upload_f32(fn);
        const int kv_dim = hp_.n_kv_heads * hp_.head_dim;
        const size_t kv_elems = size_t(hp_.n_layers) * ctx_ * kv_dim;
        kcache_ = static_cast<__half*>(dalloc(kv_elems * 2));
        vcache_ = static_cast<__half*>(dalloc(kv_elems * 2));
        cudaMemset(kcache_, 0, kv_elems * 2);
        cudaMemset(vcache_, 0, kv_elems * 2);
        kv_bytes_ = kv_elems * 4;

        // RoPE tables with the reference's own expressions (engine/src/ops_ref.cpp:204-206).
        const int half = hp_.head_dim / 2;
        std::vector<float> cs(size_t(ctx_) * half), sn(size_t(ctx_) * half);
        for (int i = 0; i < half; ++i) {
            const float freq = std::pow(hp_.rope_theta, -2.0f * i / hp_.head_dim);
            for (int pos = 0; pos < ctx_; ++pos) {
                const float angle = pos * freq;
                cs[size_t(pos) * half + i] = std::cos(angle);
                sn[size_t(pos) * half + i] = std::sin(angle);
            }
        }
        rope_cos_ = static_cast<float*>(dalloc(cs.size() * 4));
        rope_sin_ = static_cast<float*>(dalloc(sn.size() * 4));
        cudaMemcpy(rope_cos_, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(rope_sin_, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);

        // The host libm's expf exceptions, so device exps return the reference's bits (exp_table.cpp).
        {
            const std::vector<uint64_t>& slots = expf_exception_slots(&exp_note_);
            void* p = dalloc(slots.size() * 8);
            cudaMemcpy(p, slots.data(), slots.size() * 8, cudaMemcpyHostToDevice);
            exptab_.slots = static_cast<const unsigned long long*>(p);
            exptab_.mask = unsigned(slots.size() - 1);
        }
        max_chunks_ = (ctx_ + 63) / 64;

        // tensors pre-packed by export_device_layout, used when the file's layout version is this build's
        const HostTensor* lay = file_.find("b200.layout");
        const bool packed = lay && lay->dtype == DT_F32 && lay->rows * lay->cols == 1 &&
                            *reinterpret_cast<const float*>(lay->data) == float(kDeviceLayoutVersion);
        packed_tensors_ = 0;
        layers_.resize(size_t(hp_.n_layers));
        const size_t before_layers = weight_bytes_;
        for (int l = 0; l < hp_.n_layers; ++l) {
            const std::string p = "model.layers." + std::to_string(l) + ".";
            Layer& L = layers_[size_t(l)];
            L.attn_norm = upload_f32(file_.require(p + "input_layernorm.weight"));
            L.ffn_norm = upload_f32(file_.require(p + "post_attention_layernorm.weight"));
            const HostTensor &wq = file_.require(p + "self_attn.q_proj.weight"), &wk = file_.require(p + "self_attn.k_proj.weight"),
                             &wv = file_.require(p + "self_attn.v_proj.weight");
            const std::string pk = "b200.layers." + std::to_string(l) + ".";
            L.qkv = upload_packed(packed ? file_.find(pk + "qkv") : nullptr, {&wq, &wk, &wv}, 0);
            L.o = upload_matrix(file_.require(p + "self_attn.o_proj.weight"));
            L.gu = upload_packed(packed ? file_.find(pk + "gate_up") : nullptr,
                                 {&file_.require(p + "mlp.gate_proj.weight"), &file_.require(p + "mlp.up_proj.weight")}, 1);
            L.down = upload_matrix(file_.require(p + "mlp.down_proj.weight"));
            // fused bias in the q|k|v pair-interleaved order
            std::vector<float> b(size_t(L.qkv.rows), 0.f);
            if (hp_.qkv_bias) {
                // the fused bias is small: it is built here and a pre-packed copy only counts when it is the same
                b = fuse_qkv_bias({&file_.require(p + "self_attn.q_proj.bias"), &file_.require(p + "self_attn.k_proj.bias"),
                                   &file_.require(p + "self_attn.v_proj.bias")},
                                  hp_.head_dim);
                if (b.size() != size_t(L.qkv.rows)) throw std::runtime_error("qkv bias lengths do not match the q|k|v rows");
                const HostTensor* pb = packed ? file_.find(pk + "qkv_bias") : nullptr;
                if (pb && pb->dtype == DT_F32 && pb->cols == L.qkv.rows && std::memcmp(b.data(), pb->data, b.size() * 4) == 0)
                    ++packed_tensors_;
            }
            float* db = static_cast<float*>(dalloc(b.size() * 4));
            cudaMemcpy(db, b.data(), b.size() * 4, cudaMemcpyHostToDevice);
            weight_bytes_ += b.size() * 4;
            L.bqkv = db;
            QkvArgs& qa = L.qa;
            qa.W = L.qkv;
            qa.bias = db;
            qa.rope_cos = rope_cos_;
            qa.rope_sin = rope_sin_;
            qa.kcache = kcache_ + size_t(l) * ctx_ * kv_dim;
            qa.vcache = vcache_ + size_t(l) * ctx_ * kv_dim;
            qa.n_heads = hp_.n_heads;
            qa.n_kv = hp_.n_kv_heads;
            qa.head_dim = hp_.head_dim;
            qa.kv_dim = kv_dim;
            AttnArgs& aa = L.aa;
            aa.kcache = qa.kcache;
            aa.vcache = qa.vcache;
            aa.n_heads = hp_.n_heads;
            aa.n_kv = hp_.n_kv_heads;
            aa.head_dim = hp_.head_dim;
            aa.kv_dim = kv_dim;
            aa.scale = 1.0f / std::sqrt(float(hp_.head_dim));
            aa.max_chunks = max_chunks_;
            aa.exptab = exptab_;
            L.p_qkv = plan_rows(L.qkv.dtype, L.qkv.rows, L.qkv.cols, n_sm_, 2);
            L.p_o = plan_rows(L.o.dtype, L.o.rows, L.o.cols, n_sm_, 2);
            L.p_gu = plan_rows(L.gu.dtype, L.gu.rows, L.gu.cols, n_sm_, 64);
            L.p_down = plan_rows(L.down.dtype, L.down.rows, L.down.cols, n_sm_, 2);
            L.f_qkv = fuse_qkv_attn_ && qkv_attn_supported(L.qa, L.aa, nullptr);
            L.f_o = L.f_qkv && fuse_o_ && L.o.rows == hp_.dim && qkv_attn_supported(L.qa, L.aa, &L.o) &&
                    gateup_rt_supported(L.gu, L.p_gu, L.o.cols / QK);
        }
        layer_bytes_ = weight_bytes_ - before_layers + size_t(hp_.dim) * 4;

        // Exact Shortlist Head tensors (validated like engine/src/model.cpp:47-58).
        const HostTensor* q4 = file_.find("quanta.head_q4");
        const HostTensor* he = file_.find("quanta.head_err");
        if (nibble_screen) {  // the screen comes from the Q8 head itself: no file tensors, a plane of rows * cols / 2 bytes
            if (lm_head_.dtype != DT_Q8_0) return bad("the nibble-plane screen needs a Q8_0 output head");
            const size_t pb = size_t(lm_head_.rows) * lm_head_.cols / 2, eb = size_t(lm_head_.rows) * (lm_head_.cols / QK) * 2;
            uint8_t* plane = static_cast<uint8_t*>(dalloc(pb));
            __half* perr = static_cast<__half*>(dalloc(eb));
            if (launch_hi_plane(lm_head_, plane, perr, st_) != cudaSuccess) return bad("building the nibble plane failed");
            weight_bytes_ += pb + eb;
            head_err_ = perr;
            head_q4_dm_ = lm_head_;
            head_q4_dm_.dtype = DT_Q4_0;
            head_q4_dm_.q = plane;  // the Q8 head's scales stay in d
            head_q4_ = plane;
            screen_ = kScreenHi4;
        } else if (q4 || he) {
            const bool ok = q4 && he && q4->dtype == DT_Q4_0 && he->dtype == DT_F16 && lm_head_.dtype == DT_Q8_0 &&
                            q4->rows == lm_head_.rows && q4->cols == lm_head_.cols && he->rows == lm_head_.rows &&
                            he->cols == lm_head_.cols / QK;
            if (!ok) return bad("bad shortlist head tensors");
            head_q4_dm_ = upload_matrix(*q4);
            head_q4_ = head_q4_dm_.q;
            void* pe = dalloc(he->quant_bytes());
            cudaMemcpy(pe, he->data, he->quant_bytes(), cudaMemcpyHostToDevice);
            weight_bytes_ += he->quant_bytes();
            head_err_ = static_cast<const __half*>(pe);
        }

        // activations
        const int wmax = std::max(hp_.dim, hp_.ffn_dim);
        const int rmax = std::max({layers_[0].qkv.rows, 2 * hp_.ffn_dim, hp_.dim});
        X_ = static_cast<float*>(dalloc(size_t(kChunk) * hp_.dim * 4));
        Q_ = static_cast<float*>(dalloc(size_t(kChunk) * hp_.dim * 4));
        ATT_ = static_cast<float*>(dalloc(size_t(kChunk) * hp_.dim * 4));
        R_ = static_cast<float*>(dalloc(size_t(kChunk) * rmax * 4));
        OT_ = static_cast<float*>(dalloc(size_t(hp_.dim) * (layers_[0].o.cols / QK) * 4));
        if (hadamard_) HF_ = static_cast<float*>(dalloc(size_t(kChunk) * hp_.ffn_dim * 4));
        X2_ = static_cast<float*>(dalloc(size_t(hp_.dim) * 4));
        XQ_ = static_cast<int8_t*>(dalloc(size_t(kChunk) * wmax));
        DX_ = static_cast<float*>(dalloc(size_t(kChunk) * (wmax / QK) * 4));
        HQ_ = static_cast<int8_t*>(dalloc(size_t(kChunk) * hp_.ffn_dim));
        HD_ = static_cast<float*>(dalloc(size_t(kChunk) * (hp_.ffn_dim / QK) * 4));
        DXT_ = static_cast<float*>(dalloc(size_t(kChunk) * (wmax / QK) * 4));
        HDT_ = static_cast<float*>(dalloc(size_t(kChunk) * (hp_.ffn_dim / QK) * 4));
        tokens_ = static_cast<int*>(dalloc(size_t(kChunk) * 4));
        pos_ = static_cast<int*>(dalloc(16));
        // tensor-core matmul sources (a layer without them, or a driver without TMA encode, uses the CUDA cores)
        tc_act_ = make_act_maps(XQ_, DXT_, kChunk, kChunk, hp_.dim, &tm_x_) &&
                  make_act_maps(HQ_, HDT_, kChunk, kChunk, hp_.ffn_dim, &tm_h_);
        for (Layer& L : layers_)
            L.tc = tc_act_ && tc_weights(L.qkv, &L.t_qkv) && tc_weights(L.o, &L.t_o) && tc_weights(L.gu, &L.t_gu) &&
                   tc_weights(L.down, &L.t_down);

        const int V = hp_.vocab_size, nbd = hp_.dim / QK;
        hin_.xq = static_cast<int8_t*>(dalloc(size_t(hp_.dim)));
        hin_.dx = static_cast<float*>(dalloc(size_t(nbd) * 4));
        hin_.xsum = static_cast<int*>(dalloc(size_t(nbd) * 4));
        hin_.xnorm = static_cast<float*>(dalloc(size_t(nbd) * 4));
        hin_.xabs = static_cast<float*>(dalloc(size_t(nbd) * 4));
        n_lists_ = n_sm_;
        plan_full_ = plan_stream(lm_head_.dtype, V, hp_.dim, n_lists_, false, false);
        logits_ = static_cast<float*>(dalloc(size_t(V) * 4));
        coarse_ = static_cast<float*>(dalloc(size_t(V) * 4));
        upper_ = static_cast<float*>(dalloc(size_t(V) * 4));
        mark_ = static_cast<unsigned char*>(dalloc(size_t(V)));
        cudaMemset(mark_, 0, size_t(V));
        hs_ = static_cast<HeadState*>(dalloc(sizeof(HeadState)));
        cudaMemset(hs_, 0, sizeof(HeadState));
        must_ = static_cast<int*>(dalloc(size_t(ctx_ + 64) * 4));
        n_must_ = static_cast<int*>(dalloc(16));
        if (head_q4_) {
            plan_coarse_ = plan_stream(DT_Q4_0, V, hp_.dim, n_lists_, true, false);
            plan_gather_ = plan_stream(DT_Q8_0, V, hp_.dim, n_lists_, false, true);
        }
        seed_buf_ = dalloc(size_t(n_lists_) * 32 * sizeof(Cand));

        ss_ = static_cast<SamplerState*>(dalloc(sizeof(SamplerState)));
        cudaMemset(ss_, 0, sizeof(SamplerState));
        hist_ = static_cast<int*>(dalloc(size_t(ctx_ + 1) * 4));
        part_buf_ = dalloc(size_t(n_lists_) * 32 * sizeof(Cand));
        wide_ = wide_scratch_carve(dalloc(wide_scratch_bytes(V)), V);
        status_ = static_cast<unsigned*>(dalloc(16));
        cudaMemset(status_, 0, 16);
        tok_pos_ = static_cast<int*>(dalloc(size_t(kChunk) * 4));
        tok_off_ = static_cast<long long*>(dalloc(size_t(kChunk) * 8));
        head_tc_ = tc_weights(lm_head_, &t_head_);
        if (cudaStreamSynchronize(st_) != cudaSuccess) return bad("unpacking the tensor-core weights failed");
        bcand_ = dalloc(size_t(argmax_parts(hp_.vocab_size)) * kChunk * sizeof(Cand));
        bids_ = static_cast<int*>(dalloc(size_t(kChunk) * 4));
        host_tmp_.resize(size_t(V));
    } catch (const QntMissingTensor& ex) {
        file_fault_ = true;
        return bad(ex.what());
    } catch (const std::exception& ex) {
        return bad(ex.what());
    }
    cudaError_t ce = cudaDeviceSynchronize();
    if (ce != cudaSuccess) return bad(std::string("device error after load: ") + cudaGetErrorString(ce));
    return true;
}

size_t Engine::head_bytes_full() const {
    return size_t(lm_head_.rows) * (row_bytes_host(lm_head_.dtype, lm_head_.cols) + lm_head_.cols / QK * 2);
}

int Engine::debug_buffer(int what, float* out) {
    cudaStreamSynchronize(st_);
    const int dim = hp_.dim, ffn = hp_.ffn_dim;
    std::vector<int8_t> q;
    switch (what) {
        case 0: cudaMemcpy(out, Q_, size_t(dim) * 4, cudaMemcpyDeviceToHost); return dim;
        case 1: cudaMemcpy(out, ATT_, size_t(dim) * 4, cudaMemcpyDeviceToHost); return dim;
        case 2: cudaMemcpy(out, X_, size_t(dim) * 4, cudaMemcpyDeviceToHost); return dim;
        case 3:
            q.resize(size_t(ffn));
            cudaMemcpy(q.data(), HQ_, size_t(ffn), cudaMemcpyDeviceToHost);
            for (int i = 0; i < ffn; ++i) out[i] = q[size_t(i)];
            return ffn;
        case 4: cudaMemcpy(out, HD_, size_t(ffn / QK) * 4, cudaMemcpyDeviceToHost); return ffn / QK;
        case 5:
            q.resize(size_t(dim));
            cudaMemcpy(q.data(), hin_.xq, size_t(dim), cudaMemcpyDeviceToHost);
            for (int i = 0; i < dim; ++i) out[i] = q[size_t(i)];
            return dim;
    }
    return 0;
}

unsigned Engine::read_status() {
    unsigned s = 0;
    cudaMemcpy(&s, status_, 4, cudaMemcpyDeviceToHost);
    if (s) cudaMemset(status_, 0, 4);
    return s;
}

int Engine::sync_check() {
    cudaError_t e = cudaStreamSynchronize(st_);
    if (e != cudaSuccess) return cuda_fail(e, "kernel");
    unsigned s = read_status();
    if (s) {
        err_ = "device status error bits 0x" + std::to_string(s);
        return -6;
    }
    return 0;
}

// ---------------------------------------------------------------- launch sequences

#define QB_TRY(expr)                                                     \
    do {                                                                 \
        cudaError_t e_ = (expr);                                         \
        ++kernel_count_;                                                 \
        if (e_ != cudaSuccess) return cuda_fail(e_, #expr);              \
    } while (0)

int Engine::launch_layers_decode(const int* pos_dev) {
    for (const Layer& L : layers_) {
        AttnArgs aa = L.aa;  // the attention also hands o_proj its quantized input (XQ_ / DX_ are prefill scratch)
        aa.xq = XQ_;
        aa.dx = DX_;
        if (L.f_o) {  // three kernels: attention (+ q|k|v, + o_proj terms), gate|up (+ o_proj residual), down
            const OArgs oa{L.o, OT_};
            QB_TRY(launch_qkv_attn(L.qa, aa, X_, L.attn_norm, hp_.norm_eps, pos_dev, Q_, ATT_, st_, pdl_, &oa));
            QB_TRY(launch_gateup_dec(L.gu, L.p_gu, X_, L.ffn_norm, hp_.norm_eps, HQ_, HD_, exptab_, st_, pdl_, OT_,
                                     L.o.cols / QK, X2_, HF_));
            if (hadamard_) QB_TRY(launch_fwht_quant(HF_, 1, hp_.ffn_dim, HQ_, HD_, nullptr, 0, st_, pdl_));
            QB_TRY(launch_resid_dec(L.down, L.p_down, nullptr, HQ_, HD_, X_, st_, pdl_, X2_));
            continue;
        }
        if (L.f_qkv) {
            QB_TRY(launch_qkv_attn(L.qa, aa, X_, L.attn_norm, hp_.norm_eps, pos_dev, Q_, ATT_, st_, pdl_));
        } else {
            QB_TRY(launch_qkv_dec(L.qa, L.p_qkv, X_, L.attn_norm, hp_.norm_eps, pos_dev, Q_, st_, pdl_));
            QB_TRY(launch_attn(aa, Q_, pos_dev, 1, ATT_, st_, pdl_));
        }
        QB_TRY(launch_resid_dec(L.o, L.p_o, nullptr, XQ_, DX_, X_, st_, pdl_));
        QB_TRY(launch_gateup_dec(L.gu, L.p_gu, X_, L.ffn_norm, hp_.norm_eps, HQ_, HD_, exptab_, st_, pdl_, nullptr, 0, nullptr,
                                 HF_));
        if (hadamard_) QB_TRY(launch_fwht_quant(HF_, 1, hp_.ffn_dim, HQ_, HD_, nullptr, 0, st_, pdl_));
        QB_TRY(launch_resid_dec(L.down, L.p_down, nullptr, HQ_, HD_, X_, st_, pdl_));
    }
    return 0;
}

int Engine::launch_matmul(const DMat& W, const TcMap* wmap, bool ffn_in, int n, float* out, bool residual) {
    const int8_t* xq = ffn_in ? HQ_ : XQ_;
    const float* dx = ffn_in ? HD_ : DX_;
    if (wmap && n >= kTcChunkMin) {  // residual: the add onto X_ happens in the matmul's store
        QB_TRY(launch_matmul_tc(W, *wmap, ffn_in ? tm_h_ : tm_x_, n, 0, W.rows, residual ? X_ : out, W.rows, status_, st_,
                                pdl_, residual));
    } else {
        QB_TRY(launch_matmul_simt(W, xq, dx, n, 0, W.rows, out, W.rows, st_));
        if (residual) QB_TRY(launch_residual(X_, out, (long long)n * W.rows, st_, pdl_));
    }
    return 0;
}

int Engine::launch_chunk(int n, const int* pos_dev, int pos_bound, TokMap tm) {
    const int dim = hp_.dim;
    const int kv_dim = hp_.n_kv_heads * hp_.head_dim;
    for (size_t l = 0; l < layers_.size(); ++l) {
        const Layer& L = layers_[l];
        QkvArgs qa = L.qa;
        AttnArgs aa = L.aa;
        if (tm.pos) {  // the batch caches: this layer's slice of sequence 0 (tok_off adds the token's sequence)
            qa.kcache = bkcache_ + l * size_t(bctx_) * kv_dim;
            qa.vcache = bvcache_ + l * size_t(bctx_) * kv_dim;
            aa.kcache = qa.kcache;
            aa.vcache = qa.vcache;
            aa.max_chunks = (bctx_ + 63) / 64;
        }
        QB_TRY(launch_norm_quant_rows(X_, L.attn_norm, n, dim, hp_.norm_eps, XQ_, DX_, DXT_, kChunk, st_, pdl_));
        if (tc_qkv_ && L.tc && n >= kTcChunkMin && L.qkv.rows % 128 == 0) {  // bias, RoPE and the K/V stores in the matmul's epilogue
            QB_TRY(launch_matmul_tc_qkv(L.qkv, L.t_qkv, tm_x_, n, qa, pos_dev, tm, Q_, status_, st_, pdl_));
        } else {
            if (int r = launch_matmul(L.qkv, L.tc ? &L.t_qkv : nullptr, false, n, R_)) return r;
            QB_TRY(launch_qkv_epilogue(qa, R_, n, pos_dev, Q_, st_, pdl_, tm));
        }
        QuantOut qo;  // the attention quantizes its outputs for o_proj
        qo.xq = XQ_;
        qo.dx = DX_;
        qo.dxt = DXT_;
        qo.ldt = kChunk;
        QB_TRY(launch_attn_prefill(aa, Q_, pos_dev, n, pos_bound, ATT_, st_, pdl_, tm, &qo));
        if (int r = launch_matmul(L.o, L.tc ? &L.t_o : nullptr, false, n, R_, true)) return r;
        QB_TRY(launch_norm_quant_rows(X_, L.ffn_norm, n, dim, hp_.norm_eps, XQ_, DX_, DXT_, kChunk, st_, pdl_));
        if (tc_swiglu_ && L.tc && n >= kTcChunkMin && !hadamard_) {  // SwiGLU + quantize in the matmul's epilogue
            QB_TRY(launch_matmul_tc_swiglu(L.gu, L.t_gu, tm_x_, n, HQ_, HD_, HDT_, kChunk, exptab_, status_, st_, pdl_));
        } else {
            if (int r = launch_matmul(L.gu, L.tc ? &L.t_gu : nullptr, false, n, R_)) return r;
            QB_TRY(launch_swiglu_quant(R_, n, hp_.ffn_dim, HQ_, HD_, HDT_, kChunk, exptab_, st_, pdl_, HF_));
        }
        if (hadamard_) QB_TRY(launch_fwht_quant(HF_, n, hp_.ffn_dim, HQ_, HD_, HDT_, kChunk, st_, pdl_));
        if (int r = launch_matmul(L.down, L.tc ? &L.t_down : nullptr, true, n, R_, true)) return r;
    }
    return 0;
}

int Engine::launch_head(bool shortlist, int k, int n_valid, const int* must, const int* n_must_dev, int n_must_host,
                        int window, int n_list, bool penal, float penalty, bool marked) {
    if (!shortlist) {
        if (penal && !marked) QB_TRY(launch_mark(must, n_must_dev, n_must_host, window, n_valid, mark_, st_, pdl_));
        HeadFullArgs a;
        a.W = lm_head_;
        a.plan = plan_full_;
        a.n_valid = n_valid;
        a.n_list = n_list;
        a.penal = penal ? 1 : 0;
        a.penalty = penalty;
        a.mark = mark_;
        a.logits = logits_;
        a.lists = part_buf_;
        QB_TRY(launch_head_full(a, hin_, st_, pdl_));
        return 0;
    }
    ShortlistArgs a;
    a.W8 = lm_head_;
    a.W4 = head_q4_dm_;
    a.err = head_err_;
    a.screen = screen_;
    a.plan4 = plan_coarse_;
    a.plan8g = plan_gather_;
    a.k = k;
    a.n_valid = n_valid;
    a.must = must;
    a.n_must_dev = n_must_dev;
    a.n_must_host = n_must_host;
    a.window = window;
    a.mark = mark_;
    a.coarse = coarse_;
    a.upper = upper_;
    a.logits = logits_;
    a.seed_buf = seed_buf_;
    a.hs = hs_;
    a.n_list = n_list;
    a.penal = penal ? 1 : 0;
    a.penalty = penalty;
    a.lists = part_buf_;
    a.marked = marked;
    int extra = 0;
    QB_TRY(launch_shortlist(a, hin_, st_, pdl_, &extra));
    kernel_count_ += extra - 1;
    return 0;
}

int Engine::run_graph(const std::string& key, const std::function<int()>& body, bool launch) {
    if (!use_graphs_) return launch ? body() : 0;
    auto it = graphs_.find(key);
    if (it == graphs_.end()) {
        cudaGraph_t g;
        if (cudaStreamBeginCapture(st_, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return cuda_fail(cudaGetLastError(), "capture");
        const int r = body();
        cudaError_t e = cudaStreamEndCapture(st_, &g);
        if (r) return r;
        if (e != cudaSuccess) return cuda_fail(e, "end capture");
        cudaGraphExec_t ex;
        e = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return cuda_fail(e, "graph instantiate");
        it = graphs_.emplace(key, ex).first;
    }
    if (!launch) return 0;
    cudaError_t e = cudaGraphLaunch(it->second, st_);
    if (e != cudaSuccess) return cuda_fail(e, "graph launch");
    return 0;
}

// ---------------------------------------------------------------- public API

namespace {
struct HeadMode {
    bool shortlist;
    int k;
    int n_valid;
};
}  // namespace

static HeadMode head_mode(const HeadQueryC* hq, bool has_sl, int V) {
    HeadMode m{false, 0, V};
    if (hq && hq->top_k > 0 && has_sl) {
        m.shortlist = true;
        m.k = hq->top_k;
        m.n_valid = (hq->n_valid > 0 && hq->n_valid < V) ? hq->n_valid : V;
    }
    return m;
}

int Engine::forward(int token, int pos, const HeadQueryC* hq, float* out) {
    if (pos < 0 || pos >= ctx_) {
        err_ = "position exceeds context length";
        return -5;
    }
    const int V = hp_.vocab_size;
    const HeadMode hm = head_mode(hq, has_shortlist(), V);
    if (hm.shortlist && hm.k + 8 > 32) {
        err_ = "shortlist head supports top_k <= 24";
        return -4;
    }
    SamplerState st{};
    st.token = token;
    st.pos = pos;
    cudaMemcpyAsync(&ss_->pos, &st.pos, 4, cudaMemcpyHostToDevice, st_);
    cudaMemcpyAsync(&ss_->token, &st.token, 4, cudaMemcpyHostToDevice, st_);
    const int n_must = hm.shortlist ? hq->n_must : 0;
    if (n_must > ctx_ + 64) {
        err_ = "too many must ids";
        return -1;
    }
    if (n_must > 0) cudaMemcpyAsync(must_, hq->must, size_t(n_must) * 4, cudaMemcpyHostToDevice, st_);
    cudaMemcpyAsync(n_must_, &n_must, 4, cudaMemcpyHostToDevice, st_);
    const std::string key = hm.shortlist ? "fwd|sl|" + std::to_string(hm.k) + "|" + std::to_string(hm.n_valid) : "fwd|full";
    const int r = run_graph(key, [&]() -> int {
        QB_TRY(launch_embed(embed_, &ss_->token, 1, X_, status_, st_, pdl_));
        if (int rr = launch_layers_decode(&ss_->pos)) return rr;
        QB_TRY(launch_head_input(X_, final_norm_, hp_.dim, hp_.norm_eps, hin_, hs_, hm.shortlist ? 0 : V, st_, pdl_));
        return launch_head(hm.shortlist, hm.k, hm.n_valid, must_, n_must_, 0, 0, 0, false, 1.f);
    });
    if (r) return r;
    if (out) cudaMemcpyAsync(out, logits_, size_t(V) * 4, cudaMemcpyDeviceToHost, st_);
    if (int rr = sync_check()) return rr;
    if (hm.shortlist) {
        HeadState h;
        cudaMemcpy(&h, hs_, sizeof h, cudaMemcpyDeviceToHost);
        last_head_rows_ = h.rows;
    } else {
        last_head_rows_ = V;
    }
    return 0;
}

int Engine::nll(const int* ids, int n, double* total) {
    if (!ids || !total || n < 0) {
        err_ = "nll: bad argument";
        return -1;
    }
    *total = 0.0;
    if (n < 2) return 0;
    if (n > ctx_) {
        err_ = "nll: more tokens than the context holds";
        return -5;
    }
    if (!nll_acc_) nll_acc_ = static_cast<double*>(dalloc(sizeof(double)));
    const int V = hp_.vocab_size, nv = n_valid_default();
    cudaMemsetAsync(nll_acc_, 0, sizeof(double), st_);
    // Model::forward of every position but the last (full head), each followed by its target's term; one sync at the end
    for (int p = 0; p + 1 < n; ++p) {
        const int tp[2] = {ids[p], p};  // SamplerState::token, then (after n_hist) ::pos
        cudaMemcpyAsync(&ss_->token, &tp[0], 4, cudaMemcpyHostToDevice, st_);
        cudaMemcpyAsync(&ss_->pos, &tp[1], 4, cudaMemcpyHostToDevice, st_);
        const int r = run_graph("fwd|full", [&]() -> int {  // the same graph as forward() with the full head
            QB_TRY(launch_embed(embed_, &ss_->token, 1, X_, status_, st_, pdl_));
            if (int rr = launch_layers_decode(&ss_->pos)) return rr;
            QB_TRY(launch_head_input(X_, final_norm_, hp_.dim, hp_.norm_eps, hin_, hs_, V, st_, pdl_));
            return launch_head(false, 0, V, must_, n_must_, 0, 0, 0, false, 1.f);
        });
        if (r) return r;
        QB_TRY(launch_token_nll(logits_, nv, ids[p + 1], nll_acc_, st_, false));
    }
    cudaMemcpyAsync(total, nll_acc_, sizeof(double), cudaMemcpyDeviceToHost, st_);
    if (int rr = sync_check()) return rr;
    last_head_rows_ = V;
    return 0;
}

int Engine::forward_batch(const int* tokens, int n, int pos0, const HeadQueryC* hq, float* out) {
    if (n <= 0) {
        err_ = "forward_batch needs at least one token";
        return -1;
    }
    if (pos0 < 0 || pos0 + n > ctx_) {
        err_ = "position exceeds context length";
        return -5;
    }
    const int V = hp_.vocab_size;
    const HeadMode hm = head_mode(hq, has_shortlist(), V);
    if (hm.shortlist && hm.k + 8 > 32) {
        err_ = "shortlist head supports top_k <= 24";
        return -4;
    }
    int last = 0;
    for (int i = 0; i < n; i += kChunk) {
        const int m = std::min(kChunk, n - i);
        const int p = pos0 + i;
        cudaMemcpyAsync(tokens_, tokens + i, size_t(m) * 4, cudaMemcpyHostToDevice, st_);
        cudaMemcpyAsync(pos_, &p, 4, cudaMemcpyHostToDevice, st_);
        QB_TRY(launch_embed(embed_, tokens_, m, X_, status_, st_, false));
        if (int r = launch_chunk(m, pos_, p + m)) return r;
        last = m - 1;
    }
    const int n_must = hm.shortlist ? hq->n_must : 0;
    if (n_must > 0) cudaMemcpyAsync(must_, hq->must, size_t(n_must) * 4, cudaMemcpyHostToDevice, st_);
    cudaMemcpyAsync(n_must_, &n_must, 4, cudaMemcpyHostToDevice, st_);
    QB_TRY(launch_head_input(X_ + size_t(last) * hp_.dim, final_norm_, hp_.dim, hp_.norm_eps, hin_, hs_, hm.shortlist ? 0 : V, st_, pdl_));
    if (int r = launch_head(hm.shortlist, hm.k, hm.n_valid, must_, n_must_, 0, 0, 0, false, 1.f)) return r;
    if (out) cudaMemcpyAsync(out, logits_, size_t(V) * 4, cudaMemcpyDeviceToHost, st_);
    if (int rr = sync_check()) return rr;
    if (hm.shortlist) {
        HeadState h;
        cudaMemcpy(&h, hs_, sizeof h, cudaMemcpyDeviceToHost);
        last_head_rows_ = h.rows;
    } else {
        last_head_rows_ = V;
    }
    return 0;
}

int Engine::head(const HeadQueryC* hq, float* out, float* coarse, float* upper) {
    const int V = hp_.vocab_size;
    const HeadMode hm = head_mode(hq, has_shortlist(), V);
    if (hm.shortlist && hm.k + 8 > 32) {
        err_ = "shortlist head supports top_k <= 24";
        return -4;
    }
    const int n_must = hm.shortlist ? hq->n_must : 0;
    if (n_must > 0) cudaMemcpyAsync(must_, hq->must, size_t(n_must) * 4, cudaMemcpyHostToDevice, st_);
    cudaMemcpyAsync(n_must_, &n_must, 4, cudaMemcpyHostToDevice, st_);
    if (int r = launch_head(hm.shortlist, hm.k, hm.n_valid, must_, n_must_, 0, 0, 0, false, 1.f)) return r;
    if (out) cudaMemcpyAsync(out, logits_, size_t(V) * 4, cudaMemcpyDeviceToHost, st_);
    if (hm.shortlist && coarse) cudaMemcpyAsync(coarse, coarse_, size_t(V) * 4, cudaMemcpyDeviceToHost, st_);
    if (hm.shortlist && upper) cudaMemcpyAsync(upper, upper_, size_t(V) * 4, cudaMemcpyDeviceToHost, st_);
    if (int rr = sync_check()) return rr;
    if (hm.shortlist) {
        HeadState h;
        cudaMemcpy(&h, hs_, sizeof h, cudaMemcpyDeviceToHost);
        last_head_rows_ = h.rows;
    } else {
        last_head_rows_ = V;
    }
    return 0;
}

int Engine::session_begin(const int* prompt, int n_prompt, const SamplerParamsC& sp, bool use_shortlist, bool batch_prefill,
                          bool keep_rng) {
    if (n_prompt <= 0 || n_prompt >= ctx_) {  // Session::feed: pos() + n >= ctx_len is refused (session.cpp:14)
        err_ = "prompt does not fit in the context";
        return -5;
    }
    const bool greedy = sp.temperature <= 0.f;
    // top_k <= 0 (disabled) or above the 32 candidates of the fused head lists: the sorting sampler
    const bool wide = !greedy && (sp.top_k <= 0 || sp.top_k > 32);
    const int K = greedy ? 1 : sp.top_k;
    const int nv = n_valid_default();
    // Session::head_query (session.cpp:63-79) uses the shortlist with k = top_k, and the full head when k <= 0.  The
    // device shortlist keeps k + 8 <= 32 seeds; above that the full head gives the same exact top-k logits, so the
    // sampled ids do not change (only the count of exact rows does).
    const bool sl = use_shortlist && has_shortlist() && !wide && K + 8 <= 32;
    const bool penal = sp.repeat_penalty != 1.0f;
    const bool had_session = sess_.active;
    sess_ = Sess{};
    sess_.active = false;
    sess_.sp = sp;
    sess_.sl = sl;
    sess_.wide = wide;
    sess_.K = K;
    sess_.nv = nv;
    sess_.penal = penal;
    sess_.n_prompt = n_prompt;
    // session state: history = prompt, rng = seed | 1 (engine/src/sampler.cpp:15-20)
    SamplerState st{};
    st.rng = (sp.seed ? sp.seed : 0x9E3779B97F4A7C15ULL) | 1ULL;
    if (keep_rng && had_session) {  // Chat::reset keeps its Sampler: the xorshift state carries on
        if (int rr = sync_check()) return rr;
        cudaMemcpy(&st.rng, &ss_->rng, sizeof st.rng, cudaMemcpyDeviceToHost);
    }
    st.n_hist = n_prompt;
    st.pos = n_prompt - 1;
    cudaMemcpyAsync(hist_, prompt, size_t(n_prompt) * 4, cudaMemcpyHostToDevice, st_);
    cudaMemsetAsync(hs_, 0, sizeof(HeadState), st_);
    // prefill (Session::feed): head query k with must = history (when penalized)
    HeadQueryC hq;
    std::vector<int> must;
    if (sl) {
        hq.top_k = K;
        hq.n_valid = nv;
        if (penal) {
            const int from = (sp.repeat_window > 0 && n_prompt > sp.repeat_window) ? n_prompt - sp.repeat_window : 0;
            must.assign(prompt + from, prompt + n_prompt);
        }
        hq.must = must.data();
        hq.n_must = int(must.size());
    }
    if (batch_prefill) {
        if (int r = forward_batch(prompt, n_prompt, 0, sl ? &hq : nullptr, nullptr)) return r;
    } else {
        for (int i = 0; i < n_prompt; ++i) {
            if (sl && penal) {
                const int from = (sp.repeat_window > 0 && i + 1 > sp.repeat_window) ? i + 1 - sp.repeat_window : 0;
                hq.must = prompt + from;
                hq.n_must = i + 1 - from;
            }
            if (int r = forward(prompt[i], i, sl ? &hq : nullptr, nullptr)) return r;
        }
    }
    cudaMemcpyAsync(ss_, &st, sizeof st, cudaMemcpyHostToDevice, st_);  // forward() used token/pos
    // sampler stage-1 lists of the prompt's logits (the decode steps get theirs from the fused head); the sorting
    // sampler starts every step from the logits themselves
    if (!wide) {
        if (penal) QB_TRY(launch_mark(hist_, &ss_->n_hist, 0, sp.repeat_window, nv, mark_, st_, false));
        QB_TRY(launch_topk_partial(logits_, nv, K, penal ? 1 : 0, sp.repeat_penalty, mark_, part_buf_, n_lists_, st_, false));
    }
    if (int rr = sync_check()) return rr;
    sess_.active = true;
    sess_.steps = 0;
    sess_.len = n_prompt;
    return 0;
}

// decode steps per graph replay in session_step's runs
constexpr int kStepsPerGraph = 8;

int Engine::session_step(int n) {
    if (!sess_.active) {
        err_ = "no active session";
        return -1;
    }
    if (sess_.stale) {
        err_ = "the session was rewound: feed tokens before the next step";
        return -1;
    }
    const int room = ctx_ - 1 - sess_.len;
    n = std::min(n, room);
    if (n <= 0) return 0;
    const SamplerParamsC& sp = sess_.sp;
    const SamplerArgs sa{sp.temperature, sp.top_p, sp.min_p, sp.repeat_penalty, 1, exptab_};
    const bool sl = sess_.sl, penal = sess_.penal;
    const int K = sess_.K, nv = sess_.nv, V = hp_.vocab_size;
    const bool wide = sess_.wide;
    const std::string key = "gen|" + std::to_string(sl) + "|" + std::to_string(wide) + "|" + std::to_string(K) + "|" +
                            std::to_string(penal) + "|" + std::to_string(sp.repeat_window) + "|" +
                            std::to_string(sp.temperature) + "|" + std::to_string(sp.top_p) + "|" + std::to_string(sp.min_p) +
                            "|" + std::to_string(sp.repeat_penalty);
    const auto step = [&]() -> int {
        const int c0 = kernel_count_;
        if (wide) {
            // Sampler::sample over the whole logits: the penalty in place on the unique history ids, then the
            // sorting sampler; the head below only writes logits
            if (penal) {
                QB_TRY(launch_mark(hist_, &ss_->n_hist, 0, sp.repeat_window, nv, mark_, st_, pdl_));
                QB_TRY(launch_topk_partial(logits_, nv, 1, 1, sp.repeat_penalty, mark_, part_buf_, n_lists_, st_, pdl_,
                                           logits_));
            }
            int extra = 0;
            const cudaError_t e = launch_sample_wide(logits_, nv, K, sa, ss_, hist_, ctx_, wide_, st_, pdl_, &extra);
            kernel_count_ += extra;
            if (e != cudaSuccess) return cuda_fail(e, "launch_sample_wide");
            QB_TRY(launch_embed(embed_, &ss_->token, 1, X_, status_, st_, pdl_));
            if (int rr = launch_layers_decode(&ss_->pos)) return rr;
            QB_TRY(launch_head_input(X_, final_norm_, hp_.dim, hp_.norm_eps, hin_, hs_, V, st_, pdl_));
            const int rr = launch_head(false, 1, nv, nullptr, nullptr, 0, 0, 0, false, 1.0f);
            kernels_per_step_ = kernel_count_ - c0;
            return rr;
        }
        // must ids = the penalized history window (session.cpp:63-79), none without a penalty: the sampler marks
        // them for this step's head once it has drawn, so the head needs no mark kernel
        NextMarks nmk;
        if (penal) {
            nmk.mark = mark_;
            nmk.window = sp.repeat_window;
            nmk.n_valid = nv;
        }
        QB_TRY(launch_sample_final(part_buf_, n_lists_, K, sa, ss_, hist_, ctx_, st_, pdl_, &nmk));
        QB_TRY(launch_embed(embed_, &ss_->token, 1, X_, status_, st_, pdl_));
        if (int rr = launch_layers_decode(&ss_->pos)) return rr;
        QB_TRY(launch_head_input(X_, final_norm_, hp_.dim, hp_.norm_eps, hin_, hs_, sl ? 0 : V, st_, pdl_));
        const int rr = launch_head(sl, K, nv, penal ? hist_ : nullptr, penal ? &ss_->n_hist : nullptr, 0,
                                   penal ? sp.repeat_window : 0, K, penal, sp.repeat_penalty, penal);
        kernels_per_step_ = kernel_count_ - c0;
        return rr;
    };
    // Runs of kStepsPerGraph steps replay one graph of that many steps: inside it each step's first kernel starts
    // early behind the previous step's last (programmatic launch), which consecutive graph launches cannot do.  That
    // graph is captured on the first call whatever n is, so a later call never spends time instantiating it.
    const std::string key_run = key + "|x" + std::to_string(kStepsPerGraph);
    const auto run = [&]() -> int {
        for (int g = 0; g < kStepsPerGraph; ++g)
            if (int rr = step()) return rr;
        return 0;
    };
    int s = 0;
    if (use_graphs_) {
        if (int r = run_graph(key_run, run, false)) return r;
        for (; s + kStepsPerGraph <= n; s += kStepsPerGraph)
            if (int r = run_graph(key_run, run)) return r;
    }
    for (; s < n; ++s)
        if (int r = run_graph(key, step)) return r;
    sess_.steps += n;
    sess_.len += n;
    return n;
}

int Engine::session_feed(const int* ids, int n) {
    if (!sess_.active) {
        err_ = "no active session";
        return -1;
    }
    if (n <= 0) return 0;
    if (sess_.len + n >= ctx_) {  // Session::feed refuses a prompt that reaches the last position (session.cpp:14)
        err_ = "the fed tokens do not fit in the context";
        return -5;
    }
    const int L = sess_.len;
    const SamplerParamsC& sp = sess_.sp;
    cudaMemcpyAsync(hist_ + L, ids, size_t(n) * 4, cudaMemcpyHostToDevice, st_);
    // the head query of the last fed token (session.cpp:63-79): must = the penalised window of the whole history
    HeadQueryC hq;
    std::vector<int> must;
    if (sess_.sl) {
        hq.top_k = sess_.K;
        hq.n_valid = sess_.nv;
        if (sess_.penal) {
            const int total = L + n, from = (sp.repeat_window > 0 && total > sp.repeat_window) ? total - sp.repeat_window : 0;
            must.resize(size_t(total - from));
            cudaMemcpyAsync(must.data(), hist_ + from, must.size() * 4, cudaMemcpyDeviceToHost, st_);
            if (int rr = sync_check()) return rr;
        }
        hq.must = must.data();
        hq.n_must = int(must.size());
    }
    if (int r = forward_batch(ids, n, L, sess_.sl ? &hq : nullptr, nullptr)) return r;
    const int counters[2] = {L + n, L + n - 1};  // SamplerState::n_hist, ::pos (adjacent)
    cudaMemcpyAsync(&ss_->n_hist, counters, sizeof counters, cudaMemcpyHostToDevice, st_);
    if (!sess_.wide) {
        if (sess_.penal) QB_TRY(launch_mark(hist_, &ss_->n_hist, 0, sp.repeat_window, sess_.nv, mark_, st_, false));
        QB_TRY(launch_topk_partial(logits_, sess_.nv, sess_.K, sess_.penal ? 1 : 0, sp.repeat_penalty, mark_, part_buf_,
                                   n_lists_, st_, false));
    }
    if (int rr = sync_check()) return rr;
    sess_.len = L + n;
    sess_.stale = false;
    return 0;
}

int Engine::session_rewind(int n_drop) {
    if (!sess_.active || n_drop < 0 || n_drop >= sess_.len) {
        err_ = "session_rewind: needs an active session and 0 <= n_drop < its length";
        return -1;
    }
    if (n_drop == 0) return 0;
    sess_.len -= n_drop;
    const int counters[2] = {sess_.len, sess_.len - 1};
    cudaMemcpyAsync(&ss_->n_hist, counters, sizeof counters, cudaMemcpyHostToDevice, st_);
    if (int rr = sync_check()) return rr;
    sess_.stale = true;  // the logits belong to a dropped token
    return 0;
}

int Engine::session_last(int* token, int* length) {
    if (!sess_.active) {
        err_ = "no active session";
        return -1;
    }
    if (int rr = sync_check()) return rr;
    int t = -1;
    cudaMemcpy(&t, &ss_->token, 4, cudaMemcpyDeviceToHost);
    if (token) *token = t;
    if (length) *length = sess_.len;
    return 0;
}

int Engine::session_read(int* out_ids, int max_ids, GenStats* stats) {
    if (int rr = sync_check()) return rr;
    const int n = std::min(sess_.len - sess_.n_prompt, max_ids);
    if (n > 0) cudaMemcpy(out_ids, hist_ + sess_.n_prompt, size_t(n) * 4, cudaMemcpyDeviceToHost);
    if (stats) {
        HeadState h;
        cudaMemcpy(&h, hs_, sizeof h, cudaMemcpyDeviceToHost);
        // every head call of the session (session.cpp:54-61): k_head_input accumulates the previous head's rows
        stats->head_rows = h.rows_total + h.rows;
        stats->head_calls = h.calls;
    }
    return n;
}

int Engine::generate(const int* prompt, int n_prompt, const SamplerParamsC& sp, bool use_shortlist, bool batch_prefill,
                     int n_gen, int* out_ids, GenStats* stats) {
    cudaEvent_t e0, e1, e2;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventCreate(&e2);
    cudaEventRecord(e0, st_);
    int r = session_begin(prompt, n_prompt, sp, use_shortlist, batch_prefill);
    cudaEventRecord(e1, st_);
    if (r == 0) r = session_step(n_gen);
    cudaEventRecord(e2, st_);
    if (r >= 0) r = session_read(out_ids, n_gen, stats);
    float ms_pre = 0, ms_dec = 0;
    if (r >= 0) {
        cudaEventElapsedTime(&ms_pre, e0, e1);
        cudaEventElapsedTime(&ms_dec, e1, e2);
        if (stats) {
            stats->prefill_ms = ms_pre;
            stats->decode_ms = ms_dec;
        }
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaEventDestroy(e2);
    return r;
}

}  // namespace qb

namespace qb {

// ---------------------------------------------------------------- batched serving

int Engine::batch_init(int max_seqs, int ctx) {
    if (max_seqs <= 0 || ctx <= 1 || ctx > ctx_) {
        err_ = "batch_init: need max_seqs > 0 and 1 < ctx <= the model's context length";
        return -1;
    }
    if (!tc_act_ || !head_tc_) {
        err_ = "batched serving needs the tensor-core matmul (cols % 128 == 0 and a TMA-capable driver)";
        return -4;
    }
    for (const Layer& L : layers_)
        if (!L.tc) {
            err_ = "batched serving needs tensor-core sources for every layer";
            return -4;
        }
    cudaStreamSynchronize(st_);
    cudaFree(bkcache_);
    cudaFree(bvcache_);
    bkcache_ = bvcache_ = nullptr;
    const size_t kv_dim = size_t(hp_.n_kv_heads) * hp_.head_dim;
    const size_t elems = size_t(max_seqs) * hp_.n_layers * size_t(ctx) * kv_dim;
    cudaError_t e = cudaMalloc(&bkcache_, elems * 2);
    if (e == cudaSuccess) e = cudaMalloc(&bvcache_, elems * 2);
    if (e != cudaSuccess) {
        cudaFree(bkcache_);
        bkcache_ = nullptr;
        err_ = std::string("batch KV caches: ") + cudaGetErrorString(e);
        return -2;
    }
    bmax_ = max_seqs;
    bctx_ = ctx;
    blens_.assign(size_t(max_seqs), 0);
    return 0;
}

int Engine::batch_reset(int seq) {
    if (seq < 0 || seq >= bmax_) {
        err_ = "batch_reset: bad sequence id";
        return -1;
    }
    blens_[size_t(seq)] = 0;
    return 0;
}

int Engine::batch_head(int n, int* host_ids) {
    QB_TRY(launch_norm_quant_rows(X_, final_norm_, n, hp_.dim, hp_.norm_eps, XQ_, DX_, DXT_, kChunk, st_, false));
    QB_TRY(launch_matmul_tc_argmax(lm_head_, t_head_, tm_x_, n, n_valid_default(), bcand_, status_, st_, pdl_));
    QB_TRY(launch_argmax_reduce(bcand_, argmax_parts(lm_head_.rows), n, bids_, nullptr, st_));
    cudaMemcpyAsync(host_ids, bids_, size_t(n) * 4, cudaMemcpyDeviceToHost, st_);
    return sync_check();
}

int Engine::batch_prefill(int seq, const int* tokens, int n, int* next_id) {
    if (bmax_ == 0) {
        err_ = "batch_init first";
        return -1;
    }
    if (seq < 0 || seq >= bmax_ || n <= 0 || !tokens) {
        err_ = "batch_prefill: bad sequence id or tokens";
        return -1;
    }
    const int len = blens_[size_t(seq)];
    if (len + n > bctx_) {
        err_ = "batch_prefill: sequence exceeds its context";
        return -5;
    }
    const long long stride = (long long)hp_.n_layers * bctx_ * hp_.n_kv_heads * hp_.head_dim;
    int last = 0;
    for (int i = 0; i < n; i += kChunk) {
        const int m = std::min(kChunk, n - i);
        h_pos_.resize(size_t(m));
        h_off_.assign(size_t(m), stride * seq);
        for (int t = 0; t < m; ++t) h_pos_[size_t(t)] = len + i + t;
        cudaMemcpyAsync(tokens_, tokens + i, size_t(m) * 4, cudaMemcpyHostToDevice, st_);
        cudaMemcpyAsync(tok_pos_, h_pos_.data(), size_t(m) * 4, cudaMemcpyHostToDevice, st_);
        cudaMemcpyAsync(tok_off_, h_off_.data(), size_t(m) * 8, cudaMemcpyHostToDevice, st_);
        QB_TRY(launch_embed(embed_, tokens_, m, X_, status_, st_, false));
        if (int r = launch_chunk(m, pos_, len + i + m, TokMap{tok_pos_, tok_off_})) return r;
        cudaStreamSynchronize(st_);  // the host position arrays are rewritten by the next chunk
        last = m - 1;
    }
    blens_[size_t(seq)] = len + n;
    if (!next_id) return sync_check();
    // the head of the last prompt token
    if (last > 0) cudaMemcpyAsync(X_, X_ + size_t(last) * hp_.dim, size_t(hp_.dim) * 4, cudaMemcpyDeviceToDevice, st_);
    return batch_head(1, next_id);
}

int Engine::batch_decode(const int* seq_ids, const int* tokens, int n, int* next_ids) {
    if (bmax_ == 0) {
        err_ = "batch_init first";
        return -1;
    }
    if (n <= 0 || n > kChunk || !seq_ids || !tokens || !next_ids) {
        err_ = "batch_decode: need 1 <= n <= " + std::to_string(kChunk) + " sequences";
        return -1;
    }
    const long long stride = (long long)hp_.n_layers * bctx_ * hp_.n_kv_heads * hp_.head_dim;
    h_pos_.resize(size_t(n));
    h_off_.resize(size_t(n));
    std::vector<char> seen(size_t(bmax_), 0);
    int bound = 0;
    for (int i = 0; i < n; ++i) {
        const int s = seq_ids[i];
        if (s < 0 || s >= bmax_ || seen[size_t(s)]) {
            err_ = "batch_decode: sequence ids must be distinct and < max_seqs";
            return -1;
        }
        seen[size_t(s)] = 1;
        if (blens_[size_t(s)] + 1 > bctx_) {
            err_ = "batch_decode: a sequence exceeds its context";
            return -5;
        }
        h_pos_[size_t(i)] = blens_[size_t(s)];
        h_off_[size_t(i)] = stride * s;
        bound = std::max(bound, blens_[size_t(s)] + 1);
    }
    cudaMemcpyAsync(tokens_, tokens, size_t(n) * 4, cudaMemcpyHostToDevice, st_);
    cudaMemcpyAsync(tok_pos_, h_pos_.data(), size_t(n) * 4, cudaMemcpyHostToDevice, st_);
    cudaMemcpyAsync(tok_off_, h_off_.data(), size_t(n) * 8, cudaMemcpyHostToDevice, st_);
    QB_TRY(launch_embed(embed_, tokens_, n, X_, status_, st_, false));
    if (int r = launch_chunk(n, pos_, bound, TokMap{tok_pos_, tok_off_})) return r;
    if (int r = batch_head(n, next_ids)) return r;
    for (int i = 0; i < n; ++i) blens_[size_t(seq_ids[i])] += 1;
    return 0;
}

}  // namespace qb
