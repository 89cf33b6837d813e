// Model engine: the device-side replacement of quanta::Model + Session (engine/src/model.h:31-102,
// engine/src/session.h:13-80).  One Engine owns one model in HBM, one sequence's f16 KV cache and the buffers of a
// 512-token prefill chunk; forward / forward_batch / head keep the reference's contracts.  batch_* serve many
// independent sequences at once (their own KV caches), one token each per decode step, greedy.
#pragma once

#include <cuda_runtime.h>

#include <functional>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "device_layout.h"
#include "gemm_tc.h"
#include "head_kernels.h"
#include "layer_kernels.h"
#include "qnt_file.h"

namespace qb {

struct HeadQueryC {
    int top_k = 0;
    int n_valid = 0;
    const int* must = nullptr;
    int n_must = 0;
};

struct SamplerParamsC {
    float temperature = 0.7f;
    int top_k = 20;
    float top_p = 0.8f;
    float min_p = 0.0f;
    float repeat_penalty = 1.1f;
    int repeat_window = 0;
    unsigned long long seed = 0;
};

struct GenStats {
    double prefill_ms = 0, decode_ms = 0;
    long long head_rows = 0, head_calls = 0;
};

enum MatmulImpl { MM_AUTO = 0, MM_SIMT = 1, MM_TC = 2 };

class Engine {
public:
    Engine() = default;
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    // nibble_screen: screen the shortlist head with the high nibble plane of the Q8 head (kScreenHi4, plus a table of
    // the low nibbles' norms) instead of the file's quanta.head_q4 / head_err, which are then not uploaded; works for
    // files without them too.
    bool load(const std::string& path, int ctx_len, std::string* err, bool nibble_screen = false);

    // Model::forward (model.h:39): token at `pos`, logits of the head query (copied to `out` if not null).
    int forward(int token, int pos, const HeadQueryC* hq, float* out);
    // Model::forward_batch (model.h:44): n tokens at pos0.., 32-token chunks, logits of the last one.
    int forward_batch(const int* tokens, int n, int pos0, const HeadQueryC* hq, float* out);
    // Model::head (model.h:47): head of the last token again.  coarse/upper get the shortlist pass's scores.
    int head(const HeadQueryC* hq, float* out, float* coarse, float* upper);
    int last_head_rows() const { return last_head_rows_; }
    // The perplexity's sum (tools/cli/main.cpp:261-282): token by token, the full head's -log softmax of ids[p + 1]
    // after ids[0..p], summed over p < n - 1 into *total.
    int nll(const int* ids, int n, double* total);
    bool has_shortlist() const { return head_q4_ != nullptr; }

    // Session::feed + Session::generate (session.cpp:13-52) with sampling on the device: the prompt is prefilled,
    // then each step samples from the current logits, appends the id to the history and runs the next forward.
    // Returns the number of generated ids (no stop tokens), or < 0 on error.
    int generate(const int* prompt, int n_prompt, const SamplerParamsC& sp, bool use_shortlist, bool batch_prefill, int n_gen,
                 int* out_ids, GenStats* stats);

    // The same loop in pieces: prefill the prompt, run n decode steps (sample -> append -> forward, one CUDA graph
    // replay each), read the sampled ids.  generate() = begin + step(n_gen) + read.
    int session_begin(const int* prompt, int n_prompt, const SamplerParamsC& sp, bool use_shortlist, bool batch_prefill,
                      bool keep_rng = false);
    int session_step(int n);
    int session_read(int* out_ids, int max_ids, GenStats* stats);
    // Session::feed after the first (session.cpp:13-31): appends ids to the history and prefills them at the next
    // positions; the next step samples from the last one's logits.  The sampler state (xorshift) carries on.
    int session_feed(const int* ids, int n);
    // Forgets the last n_drop history tokens (a sampled stop token, which the reference never appends); a feed must
    // come before the next step.
    int session_rewind(int n_drop);
    // Waits for the queued steps: the last sampled id and the history length.
    int session_last(int* token, int* length);

    // Batched serving (greedy): up to max_seqs sequences of up to ctx positions each, KV caches of their own.
    int batch_init(int max_seqs, int ctx);
    // Prefills n prompt tokens of sequence seq (after its current length); *next_id = its greedy next token.
    int batch_prefill(int seq, const int* tokens, int n, int* next_id);
    // One decode step of n distinct sequences: tokens[i] goes to seq_ids[i] at its next position; next_ids[i] is the
    // greedy next token (std::max_element over the logits: first maximum among ids < n_valid).
    int batch_decode(const int* seq_ids, const int* tokens, int n, int* next_ids);
    int batch_reset(int seq);
    int batch_len(int seq) const { return seq >= 0 && seq < int(blens_.size()) ? blens_[size_t(seq)] : -1; }

    const HParams& hparams() const { return hp_; }
    int ctx_len() const { return ctx_; }
    int n_valid_default() const;
    size_t weight_bytes() const { return weight_bytes_; }
    size_t kv_cache_bytes() const { return kv_bytes_; }
    // copies the tensor-core matmul reads beside the weights: stage-major block scales, int8 q - 8 of Q4_0 matrices
    size_t tc_copy_bytes() const { return tc_copy_bytes_; }
    // fused tensors of the last load taken pre-packed from the file (export_device_layout), not fused at load
    int packed_tensors() const { return packed_tensors_; }
    const std::string& error() const { return err_; }
    // the last load failed on the file itself (unreadable, malformed, or a tensor missing), not on the device
    bool file_fault() const { return file_fault_; }
    void set_matmul_impl(int impl) { mm_impl_ = impl; }
    void set_use_graphs(bool on) { use_graphs_ = on; }
    void set_use_pdl(bool on) { pdl_ = on; }
    unsigned read_status();  // device error bits (and clears them)
    cudaStream_t stream() const { return st_; }
    // Per-token algorithmic bytes of one decode step's weights (layers + final norm), head excluded.
    size_t layer_weight_bytes() const { return layer_bytes_; }
    size_t head_bytes_full() const;
    // Counters of the last generate() (kernels per decode step, captured in the step graph).
    int kernels_per_step() const { return kernels_per_step_; }

    const float* logits_dev() const { return logits_; }
    // Copies an internal buffer of the last forward (token 0 of the chunk): 0 q, 1 attention output, 2 residual x,
    // 3 quantized swiglu (as float), 4 its block scales, 5 the head's quantized input.  Returns the element count.
    int debug_buffer(int what, float* out);

private:
    struct Layer {
        DMat qkv, o, gu, down;
        const float *attn_norm, *ffn_norm, *bqkv;
        QkvArgs qa;
        AttnArgs aa;
        SlicePlan p_qkv, p_o, p_gu, p_down;
        bool f_qkv = false, f_o = false;  // decode: q|k|v inside the attention kernel; o_proj folded in as well
        TcMap t_qkv{}, t_o{}, t_gu{}, t_down{};  // TMA sources of the tensor-core matmul (valid when tc)
        bool tc = false;
    };

    bool fail(const std::string& m);
    int cuda_fail(cudaError_t e, const char* what);
    void* dalloc(size_t bytes);
    DMat upload_matrix(const HostTensor& t);
    DMat upload_fused(const std::vector<const HostTensor*>& parts, int mode);
    DMat upload_packed(const HostTensor* packed, const std::vector<const HostTensor*>& parts, int mode);
    int launch_layers_decode(const int* pos_dev);
    // positions of the chunk stay below pos_bound; with tm.pos set, tokens of the batch caches (their own positions)
    int launch_chunk(int n, const int* pos_dev, int pos_bound, TokMap tm = TokMap{});
    int batch_head(int n, int* host_ids);  // greedy ids of the n rows of X_
    // Head pass: full or shortlist; n_list > 0 also produces the sampler's stage-1 lists (with the penalty of the
    // marked must ids when penal).
    // marked: the must ids were marked already (by the step's sampler), so no mark kernel runs
    int launch_head(bool shortlist, int k, int n_valid, const int* must, const int* n_must_dev, int n_must_host, int window,
                    int n_list, bool penal, float penalty, bool marked = false);
    // Prefill / batched matmul into R_: the tensor cores when the layer has TMA sources and n is large enough.
    int launch_matmul(const DMat& W, const TcMap* wmap, bool ffn_in, int n, float* out, bool residual = false);
    // TMA source of W for the tensor-core matmul (a Q4_0 matrix gets its int8 copy here); false: CUDA cores only
    bool tc_weights(const DMat& W, TcMap* map);
    // launch = false: capture and instantiate the graph (once) without running it
    int run_graph(const std::string& key, const std::function<int()>& body, bool launch = true);
    int sync_check();

    QntFile file_;
    HParams hp_;
    int ctx_ = 0, max_chunks_ = 0;
    std::string err_;
    bool file_fault_ = false;
    cudaStream_t st_ = nullptr;
    bool pdl_ = true, use_graphs_ = true;
    bool fuse_qkv_attn_ = true;  // decode: q|k|v matvec fused into the attention kernel (QNT_FUSE_QKV=0: two kernels)
    bool fuse_o_ = true;         // decode: o_proj folded into the attention + gate|up kernels (QNT_FUSE_O=0: its own kernel)
    // chunks: SwiGLU + quantize (QNT_TC_SWIGLU=1) or bias, RoPE and the K/V stores (QNT_TC_QKV=1) in the matmul's
    // epilogue instead of their own kernels.  Off: the matmul is bound by its epilogue's issue rate, and the added
    // epilogue work costs more than the launch and the f32 round trip it saves (measured at 256 sequences).
    bool tc_swiglu_ = false;
    bool tc_qkv_ = false;
    float *OT_ = nullptr, *X2_ = nullptr;  // o_proj block terms [dim][n_heads * 2] and the o_proj residual [dim]
    bool hadamard_ = false;                // FLAG_HADAMARD_DOWN file
    float* HF_ = nullptr;                  // (hadamard_) f32 SwiGLU outputs [kChunk][ffn] before the transform
    int mm_impl_ = MM_AUTO;
    int device_ = 0, n_sm_ = 148;

    std::vector<void*> allocs_;
    size_t weight_bytes_ = 0, kv_bytes_ = 0, layer_bytes_ = 0, tc_copy_bytes_ = 0;
    int packed_tensors_ = 0;

    DMat embed_{}, lm_head_{};
    const float* final_norm_ = nullptr;
    DMat head_q4_dm_{};
    const void* head_q4_ = nullptr;
    const __half* head_err_ = nullptr;
    int screen_ = kScreenQ4;  // the shortlist's screen (kScreenHi4: head_q4_dm_ is the Q8 head's high nibble plane)
    std::vector<Layer> layers_;
    float *rope_cos_ = nullptr, *rope_sin_ = nullptr;
    __half *kcache_ = nullptr, *vcache_ = nullptr;

    // activations (chunk of up to kChunk tokens)
    static constexpr int kChunk = 512;
    static constexpr int kTcChunkMin = 16;  // fewer tokens: the CUDA-core matmul
    float *X_ = nullptr, *Q_ = nullptr, *ATT_ = nullptr, *R_ = nullptr, *DX_ = nullptr, *HD_ = nullptr;
    int8_t *XQ_ = nullptr, *HQ_ = nullptr;
    float *DXT_ = nullptr, *HDT_ = nullptr;  // block scales of XQ_ / HQ_ block-major ([block][kChunk])
    TcAct tm_x_{}, tm_h_{};  // activation tiles of the tensor-core matmul (dim / ffn inputs)
    bool tc_act_ = false;
    int* tokens_ = nullptr;
    int* pos_ = nullptr;  // chunk start position (device)

    // head
    HeadIn hin_{};
    StreamPlan plan_full_{}, plan_coarse_{}, plan_gather_{};
    float *logits_ = nullptr, *coarse_ = nullptr, *upper_ = nullptr;
    unsigned char* mark_ = nullptr;
    void* seed_buf_ = nullptr;
    HeadState* hs_ = nullptr;
    int* must_ = nullptr;
    int* n_must_ = nullptr;
    int n_lists_ = 0;  // sampler stage-1 lists (one per persistent head CTA)

    // sampler / session state
    SamplerState* ss_ = nullptr;
    int* hist_ = nullptr;
    void* part_buf_ = nullptr;
    WideScratch wide_{};  // the sorting sampler's scratch (top_k 0 or > 32)
    unsigned* status_ = nullptr;
    double* nll_acc_ = nullptr;  // the perplexity's running sum

    struct Sess {
        bool active = false, sl = false, penal = false, wide = false;
        bool stale = false;  // rewound: the logits are not the last token's until the next feed
        int K = 1, nv = 0, n_prompt = 0, steps = 0;
        int len = 0;         // history length (= positions in the KV cache)
        SamplerParamsC sp;
    } sess_;
    ExpTab exptab_{};
    std::string exp_note_;
    int last_head_rows_ = 0;
    int kernels_per_step_ = 0;
    int kernel_count_ = 0;  // launches issued since the last reset (counted by the launch helpers)
    std::map<std::string, cudaGraphExec_t> graphs_;

    // batched serving
    int bmax_ = 0, bctx_ = 0;
    __half *bkcache_ = nullptr, *bvcache_ = nullptr;  // [seq][layer][bctx][kv_dim]
    std::vector<int> blens_;
    int* tok_pos_ = nullptr;              // [kChunk] device
    long long* tok_off_ = nullptr;        // [kChunk] device
    std::vector<int> h_pos_;
    std::vector<long long> h_off_;
    TcMap t_head_{};
    bool head_tc_ = false;
    void* bcand_ = nullptr;               // argmax candidates [argmax_parts(V)][kChunk]
    int* bids_ = nullptr;                 // [kChunk]
    std::vector<float> host_tmp_;
};

}  // namespace qb
