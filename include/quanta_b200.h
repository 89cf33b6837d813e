/* quanta_b200.h -- C ABI of the B200 (sm_100a) engine for Quanta.cpp's quantized-transformer hot path.
 *
 * Plain C: pointers, sizes and int status codes; no C++ or CUDA types cross this boundary (streams are void*).
 * Every entry point returns QNT_OK (0) or a negative QNT_ERR_*; qnt_last_error() gives the message of the
 * calling thread's last failure.  Exceptions never cross the ABI.
 *
 * Each declaration names the reference interface it replaces (paths inside the Quanta.cpp tree).
 */
#ifndef QUANTA_B200_H
#define QUANTA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QNT_OK 0
#define QNT_ERR_INVALID (-1)     /* bad argument / shape */
#define QNT_ERR_CUDA (-2)        /* CUDA runtime error */
#define QNT_ERR_IO (-3)          /* file open / parse error */
#define QNT_ERR_UNSUPPORTED (-4) /* valid for the reference, not implemented on the device */
#define QNT_ERR_RANGE (-5)       /* position / context overflow (reference: std::out_of_range) */
#define QNT_ERR_DEVICE (-6)      /* a kernel reported an error bit (bad token id, bounded wait timed out...) */

/* dtypes of engine/src/model_file.h:16 */
#define QNT_F32 0
#define QNT_F16 1
#define QNT_Q8_0 2
#define QNT_Q4_0 3

const char* qnt_last_error(void);
int qnt_version(void);          /* 100 * major + minor */
int qnt_device_count(void);
int qnt_set_device(int device); /* cudaSetDevice for the calling thread */

/* ---------------------------------------------------------------- ops level (engine/src/ops.h) */

typedef struct qnt_dtensor qnt_dtensor;

/* Uploads a quantized weight matrix given in the .qnt layout (quants, then fp16 scales: engine/src/model_file.h:25-38,
 * scripts/export.py:10-13) to device memory.  Replaces passing `const Tensor& W` (engine/src/ops.h:57,68).
 * When cols % 128 == 0 it also keeps what the tensor-core matmul reads: a K-step-major copy of the scales and, for
 * Q4_0, an int8 copy of q - 8 (rows * cols bytes). */
int qnt_tensor_upload(int dtype, int rows, int cols, const void* host_data, qnt_dtensor** out);
int qnt_tensor_free(qnt_dtensor* t);
int qnt_tensor_shape(const qnt_dtensor* t, int* dtype, int* rows, int* cols);

/* quantize_q8 (engine/src/ops.h:52, ops_ref.cpp:69-83) on device memory: x [n_tok][n] -> q [n_tok][n],
 * d [n_tok][n/32].  stream: a cudaStream_t or NULL. */
int qnt_quantize_q8(const float* x, int n_tok, int n, int8_t* q, float* d, void* stream);

/* MatvecQFn (engine/src/ops.h:57): out[r] = sum_b float(sum_i qW*qx) * dW * dx for r in [r0, r1); device pointers.
 * Bit-identical to matvec_q_ref (engine/src/ops_ref.cpp:85-120) built without FMA contraction. */
int qnt_matvec(const qnt_dtensor* W, const int8_t* qx, const float* dx, int r0, int r1, float* out, void* stream);

/* MatmulQFn (engine/src/ops.h:68): n activations (q [n][cols], d [n][cols/32]), out[t * ldo + r]; device pointers.
 * Per (row, token) bit-identical to qnt_matvec.  impl: 0 auto, 1 CUDA cores, 2 tensor cores (tcgen05; q and d
 * 16-byte aligned; the call makes a stream-ordered block-major copy of d with cudaMallocAsync). */
int qnt_matmul(const qnt_dtensor* W, const int8_t* qx, const float* dx, int n, int r0, int r1, float* out, int ldo,
               int impl, void* stream);

/* No reference counterpart: waits for `stream`, then reports (and clears) the status bits that the calling thread's
 * earlier qnt_matmul calls left -- QNT_ERR_DEVICE when a tensor-core wait gave up.  The host forms check it themselves. */
int qnt_ops_check(void* stream);

/* Synchronous host-pointer forms of the three calls above: the drop-in for the reference's function pointers
 * (a MatvecQFn / MatmulQFn shim passes QuantVec::q / QuantVec::d and the caller's output buffer).  Re-entrant like the
 * reference's kernels, which Model::linear calls from its thread pool on disjoint row ranges (engine/src/model.cpp:
 * 150-157): each calling thread keeps its own stream, staging buffers (device and pinned host, grown on demand, so a
 * call allocates nothing once its sizes have been seen) and kernel status word, and waits only for its own stream. */
int qnt_quantize_q8_host(const float* x, int n, int8_t* q, float* d);
int qnt_matvec_host(const qnt_dtensor* W, const int8_t* qx, const float* dx, int r0, int r1, float* out);
int qnt_matmul_host(const qnt_dtensor* W, const int8_t* qx, const float* dx, int n, int r0, int r1, float* out, int ldo,
                    int impl);

/* ---------------------------------------------------------------- model level (engine/src/model.h) */

typedef struct qnt_model qnt_model;

/* HeadQuery (engine/src/model.h:20-29). */
typedef struct qnt_head_query {
    int top_k;        /* 0 = full head */
    int n_valid;      /* ids >= n_valid are padding (0 = whole vocab) */
    const int* must;  /* ids whose logits must also be exact (e.g. penalized history) */
    int n_must;
} qnt_head_query;

/* HParams (engine/src/model_file.h:40-45). */
typedef struct qnt_hparams {
    int vocab_size, dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, max_seq;
    float rope_theta, norm_eps;
    int tied_embeddings, qkv_bias;
    uint32_t flags;
    int n_tokens;  /* tokenizer vocabulary (Tokenizer::n_tokens, engine/src/tokenizer.h:24) */
    int ctx_len;   /* KV cache positions of this model handle */
    int has_shortlist;
} qnt_hparams;

/* Model::load (engine/src/model.h:35): mmaps the .qnt, uploads every tensor once to HBM in the device layout and
 * allocates one sequence's f16 KV cache for ctx_len positions (<= 0: the file's max_seq).  flags: 0, or
 * QNT_OPEN_NIBBLE_SCREEN: the Exact Shortlist Head screens with the high nibble plane of the Q8 output head (built at
 * load: rows * cols / 2 bytes, plus an f16 norm per row and 32-block of the dropped low nibbles) instead of the
 * file's quanta.head_q4 / quanta.head_err (not uploaded), and a file
 * without those tensors gets a shortlist head too.  Exact rows, tau and the sampled ids are those of the full head
 * either way; the coarse / upper scores and the count of exact rows differ.  No reference counterpart (the
 * reference's research notes, docs/PROGRESS.md:121-130, describe the screen). */
#define QNT_OPEN_NIBBLE_SCREEN 1
int qnt_model_open(const char* path, int ctx_len, int flags, qnt_model** out);
void qnt_model_close(qnt_model* m);
int qnt_model_hparams(const qnt_model* m, qnt_hparams* out);

/* Model::forward (engine/src/model.h:39): one token at pos (positions fed in order), then the head for hq (NULL or
 * top_k <= 0: full head).  logits: host buffer of vocab_size floats or NULL.  QNT_ERR_RANGE if pos >= ctx_len. */
int qnt_model_forward(qnt_model* m, int token, int pos, const qnt_head_query* hq, float* logits);

/* Model::forward_batch (engine/src/model.h:44): n tokens at pos0..pos0+n-1 (device chunks of up to 512 tokens; the
 * results do not depend on the chunking); logits of the last. */
int qnt_model_forward_batch(qnt_model* m, const int* tokens, int n, int pos0, const qnt_head_query* hq, float* logits);

/* Model::head (engine/src/model.h:47) for the last token; coarse / upper (may be NULL) receive the shortlist pass's
 * 4-bit scores and upper bounds (Model::head_coarse / head_upper, model.h:50-51). */
int qnt_model_head(qnt_model* m, const qnt_head_query* hq, float* logits, float* coarse, float* upper);

/* The sum behind the CLI's `ppl` (tools/cli/main.cpp:261-282): Model::forward of ids[0..n-2] in order from position 0
 * (full head), and for each p the full-vocabulary -log softmax of ids[p + 1] over ids < n_tokens, summed in f64 into
 * *nll; perplexity = exp(*nll / (n - 1)).  Leaves the KV cache holding those positions. */
int qnt_model_nll(qnt_model* m, const int* ids, int n, double* nll);

/* Model::last_head_rows / has_shortlist_head / kv_cache_bytes (engine/src/model.h:48-49,58). */
int qnt_model_last_head_rows(const qnt_model* m);
int qnt_model_has_shortlist(const qnt_model* m);
size_t qnt_model_kv_cache_bytes(const qnt_model* m);
size_t qnt_model_weight_bytes(const qnt_model* m);

/* A copy of the .qnt at in_path, written to out_path, with the device's fused matrices stored pre-packed beside the
 * original tensors (which stay byte for byte, so the reference's ModelFile reads the copy as it reads the original:
 * engine/src/model_file.cpp:189-211 looks tensors up by name and ignores the rest).  Added, per layer l:
 * b200.layers.<l>.qkv (q|k|v rows pair-interleaved per head), b200.layers.<l>.gate_up (gate|up interleaved per 32
 * rows), b200.layers.<l>.qkv_bias (files with q|k|v biases), and the marker b200.layout (f32 [1], the layout
 * version).  qnt_model_open uploads those tensors as they are instead of reordering rows on the host.  The writer of
 * the format is scripts/export.py:290-315; this is its extension point (no reference counterpart).  QNT_ERR_IO if
 * in_path does not open or out_path cannot be written. */
int qnt_export_device_layout(const char* in_path, const char* out_path);
/* How many fused tensors the last qnt_model_open took pre-packed from the file (0 for a plain .qnt).  A pre-packed
 * tensor counts only when it holds the file's own rows in the fused order (shape and a sample of rows checked; the
 * q|k|v bias in full); otherwise that layer's rows are fused at load. */
int qnt_model_packed_tensors(const qnt_model* m);

/* ---------------------------------------------------------------- session + sampling (engine/src/session.h, sampler.h) */

/* SamplerParams (engine/src/sampler.h:9-18). */
typedef struct qnt_sampler_params {
    float temperature; /* <= 0: greedy */
    int top_k;         /* 0 = disabled (every candidate), as in the reference */
    float top_p, min_p;
    float repeat_penalty;
    int repeat_window; /* 0 = whole history */
    uint64_t seed;     /* 0 = fixed default seed (the reference uses the clock) */
} qnt_sampler_params;

typedef struct qnt_gen_stats {
    double prefill_ms, decode_ms;  /* device time (CUDA events) */
    long long head_rows, head_calls;
    int kernels_per_step;
} qnt_gen_stats;

#define QNT_GEN_SHORTLIST 1     /* Session::set_sampler: use the Exact Shortlist Head when the file has one */
#define QNT_GEN_BATCH_PREFILL 2 /* Session::set_batch_prefill(true) */
#define QNT_GEN_KEEP_RNG 4      /* qnt_session_begin: keep the previous session's xorshift state (a Chat::reset keeps
                                   its Sampler) instead of starting from the seed */

/* Session::feed + Session::generate (engine/src/session.cpp:13-52) with Sampler::sample (sampler.cpp:22-85) on the
 * device: prefill the prompt, then n_gen steps of sample -> append -> forward without host round trips.
 * Writes the sampled ids to out_ids and returns how many (or < 0). */
int qnt_generate(qnt_model* m, const int* prompt, int n_prompt, const qnt_sampler_params* sp, int flags, int n_gen,
                 int* out_ids, qnt_gen_stats* stats);

/* The same loop in pieces, for callers that drive decoding step by step (and for timing exactly K steps):
 * qnt_session_begin = Session::feed of the prompt (engine/src/session.cpp:13-31) with the sampler configured;
 * qnt_session_step  = n iterations of Session::generate's loop body (session.cpp:45-53), queued on the model's stream
 *                     (returns without waiting; at most ctx_len - 1 positions in total);
 * qnt_session_read  = waits for the queued steps and copies the sampled ids (returns how many). */
int qnt_session_begin(qnt_model* m, const int* prompt, int n_prompt, const qnt_sampler_params* sp, int flags);
int qnt_session_step(qnt_model* m, int n);
int qnt_session_read(qnt_model* m, int* out_ids, int max_ids, qnt_gen_stats* stats);

/* The rest of Session (engine/src/session.cpp:13-52) for multi-turn use (Chat::reply, session.cpp:94-118):
 *   qnt_session_feed    Session::feed after the first: appends n ids to the history and prefills them at the next
 *                       positions (the same results as feeding them with the first prompt); the sampler state carries on.
 *   qnt_session_rewind  forgets the last n_drop history tokens -- a sampled stop token, which the reference never
 *                       appends (session.cpp:41-42); the next call on the session must be a feed.
 *   qnt_session_last    waits for the queued steps; *token = the last sampled id, *length = the history length. */
int qnt_session_feed(qnt_model* m, const int* ids, int n);
int qnt_session_rewind(qnt_model* m, int n_drop);
int qnt_session_last(qnt_model* m, int* token, int* length);

/* Text <-> ids (engine/src/tokenizer.h:15-39): byte-level BPE over the .qnt's tokenizer section, on the host (no GPU).
 *   qnt_tokenizer_open  Tokenizer(ModelFile::tokenizer()): QNT_ERR_IO for an unreadable file or a vocabulary without
 *                       all 256 byte tokens
 *   qnt_tokenize        Tokenizer::encode (special literals such as "<|im_start|>" recognised): returns the id count and
 *                       writes at most max_ids of them
 *   qnt_token_piece     Tokenizer::decode(id): the raw bytes (possibly part of a UTF-8 sequence); returns their count and
 *                       writes at most cap of them (an unknown id has none)
 *   qnt_token_id        Tokenizer::token_id: a special token's id, or -1 */
typedef struct qnt_tokenizer qnt_tokenizer;
int qnt_tokenizer_open(const char* path, qnt_tokenizer** out);
void qnt_tokenizer_free(qnt_tokenizer* t);
int qnt_tokenizer_n_tokens(const qnt_tokenizer* t);
int qnt_tokenize(const qnt_tokenizer* t, const char* text, size_t len, int* ids, int max_ids);
int qnt_token_piece(const qnt_tokenizer* t, int id, char* buf, int cap);
int qnt_token_id(const qnt_tokenizer* t, const char* literal);

/* Batched serving of many independent sequences on one model (the multi-sequence API qnt_prefill_batch /
 * qnt_decode_batch of the drop-in boundary; the reference serves one Session at a time, engine/src/session.cpp:13-52).
 * Each sequence has its own f16 KV cache; a decode step advances n distinct sequences by one token each through the
 * tensor-core matmul (tokens as the matmul's N), and the greedy head is one tensor-core pass over the Q8 lm_head with
 * the argmax fused (Sampler::sample at temperature 0: the first maximum over ids < n_valid).
 *   qnt_batch_init     allocates the caches of max_seqs sequences of ctx_len positions (lengths reset to 0)
 *   qnt_prefill_batch  feeds n prompt tokens to sequence seq; *next_id = its greedy next token (may be NULL)
 *   qnt_decode_batch   n <= 512 distinct sequences, tokens[i] appended to seq_ids[i]; next_ids[i] its greedy next token
 *   qnt_batch_reset    forgets sequence seq (length 0) */
int qnt_batch_init(qnt_model* m, int max_seqs, int ctx_len);
int qnt_prefill_batch(qnt_model* m, int seq, const int* tokens, int n, int* next_id);
int qnt_decode_batch(qnt_model* m, const int* seq_ids, const int* tokens, int n, int* next_ids);
int qnt_batch_reset(qnt_model* m, int seq);

/* Sampler (engine/src/sampler.h:20-38): Sampler::sample (sampler.cpp:22-85) on logits that are already in device
 * memory -- repetition penalty -> greedy argmax (first max) or top-k -> softmax(T) -> min-p -> top-p -> xorshift64*
 * draw, with the reference's float operations, so the same logits, history and seed give the same ids.
 *   qnt_sampler_create  = Sampler(const SamplerParams&): the xorshift state starts at (seed ? seed : fixed) | 1, on the
 *                         current device.  Any top_k: up to 32 the candidates come from per-CTA lists; top_k 0 (disabled)
 *                         or above 32 sorts every logit below n_valid on the device (scratch of 16 B per id, allocated
 *                         on first use and kept by the sampler).
 *   qnt_sampler_sample  = Sampler::sample(float* logits, int n_valid, const std::vector<int>& history): `logits` is a
 *                         DEVICE array of at least n_valid floats and is edited in place like the reference's (the
 *                         penalised ids); `history` is a host array of n_history ids.  Work is queued on `stream`
 *                         (a cudaStream_t, NULL = legacy default); the call waits for it and writes the id to *token.
 *   qnt_sampler_free    = ~Sampler. */
typedef struct qnt_sampler qnt_sampler;
int qnt_sampler_create(const qnt_sampler_params* sp, qnt_sampler** out);
int qnt_sampler_sample(qnt_sampler* s, float* logits, int n_valid, const int* history, int n_history, int* token,
                       void* stream);
void qnt_sampler_free(qnt_sampler* s);

/* No counterpart in the reference: qnt_sampler_sample without a sampler object and without allocating memory, for
 * callers that cannot allocate -- a serving process whose device memory is reserved up front by its own pool (weights
 * and KV pages), where a cudaMalloc fails or fragments that pool, and a token loop that must not stall other streams,
 * as cudaMalloc / cudaFree can synchronise the device.  Same kernels and results as qnt_sampler_sample.
 *   *rng_state: the xorshift64* state, in/out; start it at (seed ? seed : any nonzero) | 1 as Sampler's constructor
 *               does (sampler.cpp:10-13); each call advances it exactly like the sampler object's.
 *   Limits: n_valid <= 262144, n_history <= 32768, 1 <= top_k <= 32 when temperature > 0; larger sizes return
 *           QNT_ERR_INVALID with the limit in qnt_last_error().
 *   Scratch: one static device array of 459,008 bytes per device (sampler state, candidate lists, history copy and
 *            penalty marks) plus a static 4 MiB copy of the host exp table.  The marks must be all zero when a call
 *            starts: they start zeroed, every completed call clears the ones it set, and a call that fails after
 *            setting them clears them (a stream-ordered memset) before it returns its error.  Calls whose GPU work
 *            overlaps (other host threads, or other streams) share that scratch and race: serialise them.
 *   The first call on each device does the set-up, with that device current: cudaGetSymbolAddress of the scratch and
 *            of the table, and a synchronous copy of the exp table into it.  Make that first call before any stream
 *            capture begins.  Every call copies its parameters and history through pageable host memory, waits for
 *            its stream (cudaStreamSynchronize) and writes the id to *token. */
int qnt_sampler_sample_noalloc(const qnt_sampler_params* sp, uint64_t* rng_state, float* logits, int n_valid,
                               const int* history, int n_history, int* token, void* stream);

/* Diagnostics (no reference counterpart): copies an internal buffer of the last forward as floats -- 0 roped q,
 * 1 attention output, 2 residual x (of the last layer, before the final norm), 3 quantized SwiGLU output, 4 its block
 * scales, 5 the head's quantized input.  Returns the element count. */
int qnt_model_debug_buffer(qnt_model* m, int what, float* out);

/* The cudaStream_t (as void*) every call on this model is queued on: lets a caller record CUDA events around
 * qnt_session_step for device timing. */
void* qnt_model_stream(const qnt_model* m);

/* Diagnostics (no reference counterpart): the dense int8 tensor-core rate of the current GPU, measured -- every SM
 * issues 4 * iters back-to-back tcgen05.mma.kind::i8 (M 128, N 256, K 32) on operands resident in shared memory;
 * *tops = int8 TOP/s over the slowest SM.  The roofline denominator of the tensor-core matmul. */
int qnt_bench_mma_i8(int iters, double* tops);

/* Diagnostics (no reference counterpart): runs the tensor-core matmul's bounded wait on an mbarrier that nothing
 * completes, with `limit` tries (1..2^20; each try may sleep up to 20 us), on `stream`.  The wait runs out, the kernel
 * records the timeout in the calling thread's status word and returns, and the call reports it as QNT_ERR_DEVICE --
 * the path a real timeout takes, shown without a fault; the context stays usable. */
int qnt_wait_probe(unsigned limit, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QUANTA_B200_H */
