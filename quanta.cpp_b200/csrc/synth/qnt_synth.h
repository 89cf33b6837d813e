// Seeded random-init .qnt writer (synthetic stand-in for scripts/export.py).  See qnt_synth.cpp.
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct qnt_synth_cfg {
    int vocab_size, dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, max_seq;
    float rope_theta, norm_eps;
    int mlp_q4;      // 1: MLP matrices as GPTQ-sym int4 (Q4_0), attention stays Q8_0 ("q4mix"); 0: all Q8_0
    int q4_group;    // scale group of the int4 codes in columns (128 = g128; a multiple of 32)
    int shortlist;   // 1: add quanta.head_q4 / quanta.head_err (Exact Shortlist Head)
    int n_tokens;    // tokenizer vocabulary (<= vocab_size; rows beyond it are padding); 0 = vocab_size
    float w_std;     // weight std (0 = 0.02)
    uint64_t seed;
    int n_threads;   // 0 = all hardware threads
    unsigned flags;  // header flags (1 = FLAG_HADAMARD_DOWN: the reference transforms the SwiGLU output before down)
    const unsigned char* tok_blob;  // a complete tokenizer section to write instead of the synthetic byte vocabulary
    uint64_t tok_len;               // (its vocabulary size must equal n_tokens; 0 / null: the synthetic one)
} qnt_synth_cfg;

int qnt_synth_write(const char* path, const qnt_synth_cfg* cfg);  // 0 on success
const char* qnt_synth_last_error(void);

#ifdef __cplusplus
}
#endif
