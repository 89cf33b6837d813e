/* qnt_oracle.c -- CPU restatement of Quanta.cpp's quantized-transformer path, in plain C.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product).  Built by oracle/oracle.mk into
 * oracle/_build/libqnt_oracle.so; loaded by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg.
 * Pinned against the reference compiled from its own sources (oracle/_ref, oracle/Makefile): the tests require
 * identical bits on the same inputs.  Built, like the reference checker, without FMA contraction so every float
 * expression rounds exactly as written.
 *
 * Single-threaded on purpose (the reference's ThreadPool only splits independent rows/heads, which does not change
 * any value).  Each function cites the reference lines it restates.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <fcntl.h>
#include <unistd.h>

#define QK 32
enum { DT_F32 = 0, DT_F16 = 1, DT_Q8_0 = 2, DT_Q4_0 = 3 };

/* ---------------------------------------------------------------- scalar helpers */

/* fp16 bits -> float (engine/src/ops.h:15-40): normal, subnormal (renormalized), inf/nan. */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int ex = 127 - 15 + 1;
            while (!(m & 0x400u)) {
                m <<= 1;
                --ex;
            }
            bits = sign | ((uint32_t)ex << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 127 - 15) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t f32_to_f16(float f) { /* round to nearest even, as the reference's _Float16(float) store */
    _Float16 h = (_Float16)f;
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}

/* quantize_q8 (engine/src/ops_ref.cpp:69-83). */
void orc_quantize_q8(const float* x, int n, int8_t* q, float* d) {
    for (int b = 0; b < n / QK; ++b) {
        const float* xb = x + b * QK;
        float amax = 0.f;
        for (int i = 0; i < QK; ++i) amax = fmaxf(amax, fabsf(xb[i]));
        const float dd = amax / 127.f;
        const float inv = dd > 0 ? 1.f / dd : 0.f;
        for (int i = 0; i < QK; ++i) q[b * QK + i] = (int8_t)lroundf(xb[i] * inv);
        d[b] = dd;
    }
}

/* matvec_q_ref (engine/src/ops_ref.cpp:85-120): out[r] = sum_b float(int32 block sum) * dW_b * dx_b in block order. */
void orc_matvec_q(int dtype, int rows, int cols, const uint8_t* data, const int8_t* qx, const float* dx, int r0, int r1,
                  float* out) {
    const int nb = cols / QK;
    const size_t qbytes = dtype == DT_Q8_0 ? (size_t)rows * cols : (size_t)rows * cols / 2;
    const uint16_t* dw = (const uint16_t*)(data + qbytes);
    for (int r = r0; r < r1; ++r) {
        float acc = 0.f;
        for (int b = 0; b < nb; ++b) {
            int32_t s = 0;
            if (dtype == DT_Q8_0) {
                const int8_t* w = (const int8_t*)data + (size_t)r * cols + (size_t)b * QK;
                for (int i = 0; i < QK; ++i) s += (int32_t)w[i] * qx[b * QK + i];
            } else {
                const uint8_t* w = data + ((size_t)r * cols + (size_t)b * QK) / 2;
                for (int j = 0; j < QK / 2; ++j) {
                    s += ((int32_t)(w[j] & 0xF) - 8) * qx[b * QK + j];
                    s += ((int32_t)(w[j] >> 4) - 8) * qx[b * QK + j + QK / 2];
                }
            }
            acc += (float)s * orc_f16_to_f32(dw[(size_t)r * nb + b]) * dx[b];
        }
        out[r] = acc;
    }
}

/* matmul_q_ref (engine/src/ops_ref.cpp:122-160) is bit-identical to matvec per (row, token). */
void orc_matmul_q(int dtype, int rows, int cols, const uint8_t* data, const int8_t* qx, const float* dx, int n, int r0,
                  int r1, float* out, int ldo) {
    float* tmp = malloc(sizeof(float) * (size_t)rows);
    for (int t = 0; t < n; ++t) {
        orc_matvec_q(dtype, rows, cols, data, qx + (size_t)t * cols, dx + (size_t)t * (cols / QK), r0, r1, tmp);
        for (int r = r0; r < r1; ++r) out[(size_t)t * ldo + r] = tmp[r];
    }
    free(tmp);
}

/* get_row (engine/src/ops_ref.cpp:162-192), quantized rows. */
static void get_row(float* out, int dtype, int cols, const uint8_t* data, size_t qbytes, int row) {
    const uint16_t* dw = (const uint16_t*)(data + qbytes);
    const int nb = cols / QK;
    if (dtype == DT_Q8_0) {
        const int8_t* q = (const int8_t*)data + (size_t)row * cols;
        for (int i = 0; i < cols; ++i) out[i] = q[i] * orc_f16_to_f32(dw[(size_t)row * nb + i / QK]);
    } else {
        const uint8_t* q = data + (size_t)row * cols / 2;
        for (int b = 0; b < nb; ++b) {
            const float s = orc_f16_to_f32(dw[(size_t)row * nb + b]);
            for (int j = 0; j < QK / 2; ++j) {
                out[b * QK + j] = ((int)(q[b * QK / 2 + j] & 0xF) - 8) * s;
                out[b * QK + j + QK / 2] = ((int)(q[b * QK / 2 + j] >> 4) - 8) * s;
            }
        }
    }
}

/* rmsnorm (engine/src/ops_ref.cpp:194-199). */
static void rmsnorm(float* out, const float* x, const float* w, int n, float eps) {
    float ss = 0.f;
    for (int i = 0; i < n; ++i) ss += x[i] * x[i];
    const float scale = 1.0f / sqrtf(ss / n + eps);
    for (int i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

/* rope, NeoX rotate-half (engine/src/ops_ref.cpp:201-214). */
static void rope(float* v, int n_heads, int hd, int pos, float theta) {
    const int half = hd / 2;
    for (int i = 0; i < half; ++i) {
        const float freq = powf(theta, -2.0f * i / hd);
        const float angle = pos * freq;
        const float c = cosf(angle), s = sinf(angle);
        for (int h = 0; h < n_heads; ++h) {
            float* p = v + h * hd;
            const float a = p[i], b = p[i + half];
            p[i] = a * c - b * s;
            p[i + half] = b * c + a * s;
        }
    }
}

/* exp as the reference evaluates it (std::exp on float = expf).  orc_set_exp_double(1) switches to the double exp
 * rounded once to float, to measure how much the libm's last-bit choices matter. */
static int g_exp_double = 0;
void orc_set_exp_double(int on) { g_exp_double = on; }
static float ref_expf(float x) { return g_exp_double ? (float)exp((double)x) : expf(x); }

/* softmax (engine/src/ops_ref.cpp:216-226). */
static void softmax(float* x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; ++i) mx = x[i] > mx ? x[i] : mx;
    float sum = 0.f;
    for (int i = 0; i < n; ++i) {
        x[i] = ref_expf(x[i] - mx);
        sum += x[i];
    }
    const float inv = 1.0f / sum;
    for (int i = 0; i < n; ++i) x[i] *= inv;
}

/* ---------------------------------------------------------------- .qnt reader (engine/src/model_file.cpp:149-211) */

typedef struct {
    char name[96];
    int dtype, rows, cols;
    const uint8_t* data;
} OTensor;

typedef struct {
    int vocab, dim, n_layers, n_heads, n_kv, hd, ffn, max_seq, n_tokens;
    float theta, eps;
    int tied, qkv_bias;
    uint32_t flags;
    const uint8_t* base;
    size_t size;
    OTensor* t;
    int nt;
    int ctx;
    /* layer tensors */
    const OTensor *embed, *final_norm, *lm_head, *head_q4, *head_err;
    const OTensor** L; /* 12 per layer */
    /* state */
    float *x, *xb, *xb2, *q, *k, *v, *att, *hb, *hb2, *logits, *coarse, *upper, *xnorm;
    int8_t *xq, *hq;
    float *xd, *hd_;
    uint16_t *kc, *vc;
    uint8_t* must_mark;
    int last_head_rows;
    /* snapshots of the last layer of the last forward (debugging aid for the device path) */
    float *dbg_q, *dbg_att, *dbg_x;
} OModel;

static size_t quant_bytes(const OTensor* t) {
    const size_t n = (size_t)t->rows * t->cols;
    switch (t->dtype) {
        case DT_F32: return n * 4;
        case DT_F16: return n * 2;
        case DT_Q8_0: return n;
        default: return n / 2;
    }
}

static const OTensor* find(const OModel* m, const char* name) {
    for (int i = 0; i < m->nt; ++i)
        if (strcmp(m->t[i].name, name) == 0) return &m->t[i];
    return NULL;
}

typedef struct {
    const uint8_t *p, *end;
    int bad;
} Rd;
static uint32_t rd_u32(Rd* r) {
    if (r->end - r->p < 4) {
        r->bad = 1;
        return 0;
    }
    uint32_t v;
    memcpy(&v, r->p, 4);
    r->p += 4;
    return v;
}
static uint64_t rd_u64(Rd* r) {
    if (r->end - r->p < 8) {
        r->bad = 1;
        return 0;
    }
    uint64_t v;
    memcpy(&v, r->p, 8);
    r->p += 8;
    return v;
}
static void rd_skip(Rd* r, size_t n) {
    if ((size_t)(r->end - r->p) < n) {
        r->bad = 1;
        return;
    }
    r->p += n;
}

void orc_model_close(OModel* m);

OModel* orc_model_open(const char* path, int ctx, char* err, int errlen) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) {
        snprintf(err, (size_t)errlen, "cannot open %s", path);
        return NULL;
    }
    struct stat st;
    fstat(fd, &st);
    void* p = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (p == MAP_FAILED) {
        snprintf(err, (size_t)errlen, "mmap failed");
        return NULL;
    }
    OModel* m = calloc(1, sizeof *m);
    m->base = p;
    m->size = (size_t)st.st_size;
    Rd r = {m->base, m->base + m->size, 0};
    if (m->size < 4 || memcmp(r.p, "QNT1", 4) != 0) {
        snprintf(err, (size_t)errlen, "bad magic");
        orc_model_close(m);
        return NULL;
    }
    r.p += 4;
    const uint32_t version = rd_u32(&r);
    m->vocab = (int)rd_u32(&r);
    m->dim = (int)rd_u32(&r);
    m->n_layers = (int)rd_u32(&r);
    m->n_heads = (int)rd_u32(&r);
    m->n_kv = (int)rd_u32(&r);
    m->hd = (int)rd_u32(&r);
    m->ffn = (int)rd_u32(&r);
    m->max_seq = (int)rd_u32(&r);
    uint32_t u = rd_u32(&r);
    memcpy(&m->theta, &u, 4);
    u = rd_u32(&r);
    memcpy(&m->eps, &u, 4);
    m->tied = rd_u32(&r) != 0;
    m->qkv_bias = rd_u32(&r) != 0;
    m->flags = version >= 2 ? rd_u32(&r) : 0;
    if ((m->flags & 1u) && m->ffn % 256 != 0) { /* engine/src/model.cpp:39-42 */
        snprintf(err, (size_t)errlen, "FLAG_HADAMARD_DOWN needs ffn_dim %% 256 == 0");
        orc_model_close(m);
        return NULL;
    }
    const uint32_t tok_len = rd_u32(&r);
    if (!r.bad) {
        Rd t = {r.p, r.p + tok_len, 0};
        m->n_tokens = (int)rd_u32(&t);
    }
    rd_skip(&r, tok_len);
    m->nt = (int)rd_u32(&r);
    m->t = calloc((size_t)(m->nt > 0 ? m->nt : 1), sizeof(OTensor));
    for (int i = 0; i < m->nt && !r.bad; ++i) {
        const uint32_t n = rd_u32(&r);
        if (n >= sizeof m->t[i].name || (size_t)(r.end - r.p) < n) {
            r.bad = 1;
            break;
        }
        memcpy(m->t[i].name, r.p, n);
        r.p += n;
        m->t[i].dtype = (int)rd_u32(&r);
        const uint32_t nd = rd_u32(&r);
        if (nd == 1) {
            m->t[i].rows = 1;
            m->t[i].cols = (int)rd_u32(&r);
        } else {
            m->t[i].rows = (int)rd_u32(&r);
            m->t[i].cols = (int)rd_u32(&r);
        }
        const uint64_t off = rd_u64(&r);
        size_t total = quant_bytes(&m->t[i]);
        if (m->t[i].dtype >= DT_Q8_0) total += (size_t)m->t[i].rows * m->t[i].cols / QK * 2;
        if (off + total > m->size) r.bad = 1;
        m->t[i].data = m->base + off;
    }
    if (r.bad) {
        snprintf(err, (size_t)errlen, "model file truncated or out of bounds");
        orc_model_close(m);
        return NULL;
    }
    m->embed = find(m, "model.embed_tokens.weight");
    m->final_norm = find(m, "model.norm.weight");
    m->lm_head = m->tied ? m->embed : find(m, "lm_head.weight");
    m->head_q4 = find(m, "quanta.head_q4");
    m->head_err = find(m, "quanta.head_err");
    m->L = calloc((size_t)m->n_layers * 12, sizeof(OTensor*));
    static const char* names[12] = {"input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
                                    "self_attn.v_proj.weight", "self_attn.o_proj.weight", "self_attn.q_proj.bias",
                                    "self_attn.k_proj.bias", "self_attn.v_proj.bias", "post_attention_layernorm.weight",
                                    "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"};
    for (int l = 0; l < m->n_layers; ++l)
        for (int k = 0; k < 12; ++k) {
            char nm[128];
            snprintf(nm, sizeof nm, "model.layers.%d.%s", l, names[k]);
            m->L[l * 12 + k] = find(m, nm);
            if (!m->L[l * 12 + k] && !(k >= 5 && k <= 7 && !m->qkv_bias)) {
                snprintf(err, (size_t)errlen, "missing tensor: %s", nm);
                orc_model_close(m);
                return NULL;
            }
        }
    if (!m->embed || !m->final_norm || !m->lm_head) {
        snprintf(err, (size_t)errlen, "missing tensor");
        orc_model_close(m);
        return NULL;
    }
    m->ctx = (ctx > 0 && ctx < m->max_seq) ? ctx : m->max_seq;
    const int qd = m->n_heads * m->hd, kvd = m->n_kv * m->hd, V = m->vocab;
    m->x = calloc((size_t)m->dim, 4);
    m->xb = calloc((size_t)m->dim, 4);
    m->xb2 = calloc((size_t)m->dim, 4);
    m->q = calloc((size_t)qd, 4);
    m->k = calloc((size_t)kvd, 4);
    m->v = calloc((size_t)kvd, 4);
    m->att = calloc((size_t)m->n_heads * m->ctx, 4);
    m->hb = calloc((size_t)m->ffn, 4);
    m->hb2 = calloc((size_t)m->ffn, 4);
    m->logits = calloc((size_t)V, 4);
    m->coarse = calloc((size_t)V, 4);
    m->upper = calloc((size_t)V, 4);
    m->xnorm = calloc((size_t)(m->dim / QK), 4);
    m->xq = calloc((size_t)m->dim, 1);
    m->xd = calloc((size_t)(m->dim / QK), 4);
    m->hq = calloc((size_t)m->ffn, 1);
    m->hd_ = calloc((size_t)(m->ffn / QK), 4);
    m->kc = calloc((size_t)m->n_layers * m->ctx * kvd, 2);
    m->vc = calloc((size_t)m->n_layers * m->ctx * kvd, 2);
    m->must_mark = calloc((size_t)V, 1);
    m->dbg_q = calloc((size_t)qd, 4);
    m->dbg_att = calloc((size_t)m->dim, 4);
    m->dbg_x = calloc((size_t)m->dim, 4);
    return m;
}

void orc_model_close(OModel* m) {
    if (!m) return;
    if (m->base) munmap((void*)m->base, m->size);
    free(m->t);
    free(m->L);
    float* fs[] = {m->x, m->xb, m->xb2, m->q, m->k, m->v, m->att, m->hb, m->hb2, m->logits, m->coarse, m->upper, m->xnorm, m->xd, m->hd_};
    for (size_t i = 0; i < sizeof fs / sizeof fs[0]; ++i) free(fs[i]);
    free(m->xq);
    free(m->hq);
    free(m->kc);
    free(m->vc);
    free(m->must_mark);
    free(m->dbg_q);
    free(m->dbg_att);
    free(m->dbg_x);
    free(m);
}

int orc_vocab(const OModel* m) { return m->vocab; }

/* Copies a snapshot of the last forward: 0 q (roped, last layer), 1 attention output (last layer), 2 residual x before
 * the final norm, 3 quantized swiglu of the last layer (as float), 4 its block scales, 5 the head's quantized input. */
int orc_debug(const OModel* m, int what, float* out) {
    switch (what) {
        case 0: memcpy(out, m->dbg_q, sizeof(float) * (size_t)(m->n_heads * m->hd)); return m->n_heads * m->hd;
        case 1: memcpy(out, m->dbg_att, sizeof(float) * (size_t)m->dim); return m->dim;
        case 2: memcpy(out, m->dbg_x, sizeof(float) * (size_t)m->dim); return m->dim;
        case 3: for (int i = 0; i < m->ffn; ++i) out[i] = m->hq[i]; return m->ffn;
        case 4: memcpy(out, m->hd_, sizeof(float) * (size_t)(m->ffn / QK)); return m->ffn / QK;
        case 5: for (int i = 0; i < m->dim; ++i) out[i] = m->xq[i]; return m->dim;
    }
    return 0;
}
int orc_n_tokens(const OModel* m) { return m->n_tokens; }
int orc_last_head_rows(const OModel* m) { return m->last_head_rows; }

static void linear(OModel* m, float* out, const OTensor* W, const int8_t* xq, const float* xd) {
    orc_matvec_q(W->dtype, W->rows, W->cols, W->data, xq, xd, 0, W->rows, out);
}

static void add_bias(float* v, const OTensor* b) { /* engine/src/model.cpp:159-163 */
    if (!b) return;
    const float* bb = (const float*)b->data;
    for (int i = 0; i < b->cols; ++i) v[i] += bb[i];
}

/* attend<_Float16> (engine/src/model.cpp:115-137). */
/* Block Walsh-Hadamard transform in place (engine/src/ops_ref.cpp:228-241): in each block, stages h = 1, 2, ..,
 * block / 2 replace (v[j], v[j + h]) by (v[j] + v[j + h], v[j] - v[j + h]) within 2h-blocks, then scale by
 * 1 / sqrt(block). */
static void fwht_blocks(float* x, int n, int block) {
    const float norm = 1.0f / sqrtf((float)block);
    for (int b0 = 0; b0 < n; b0 += block) {
        float* v = x + b0;
        for (int h = 1; h < block; h *= 2)
            for (int i = 0; i < block; i += 2 * h)
                for (int j = i; j < i + h; ++j) {
                    const float a = v[j], c = v[j + h];
                    v[j] = a + c;
                    v[j + h] = a - c;
                }
        for (int i = 0; i < block; ++i) v[i] *= norm;
    }
}

static void attend(OModel* m, const uint16_t* kc, const uint16_t* vc, int pos) {
    const int hd = m->hd, kvd = m->n_kv * hd, group = m->n_heads / m->n_kv;
    const float scale = 1.0f / sqrtf((float)hd);
    for (int h = 0; h < m->n_heads; ++h) {
        const float* qh = m->q + h * hd;
        const int kvh = h / group;
        float* att = m->att + (size_t)h * m->ctx;
        for (int t = 0; t <= pos; ++t) {
            const uint16_t* kt = kc + (size_t)t * kvd + kvh * hd;
            float s = 0.f;
            for (int i = 0; i < hd; ++i) s += qh[i] * orc_f16_to_f32(kt[i]);
            att[t] = s * scale;
        }
        softmax(att, pos + 1);
        float* out = m->xb + h * hd;
        for (int i = 0; i < hd; ++i) out[i] = 0.f;
        for (int t = 0; t <= pos; ++t) {
            const uint16_t* vt = vc + (size_t)t * kvd + kvh * hd;
            const float a = att[t];
            for (int i = 0; i < hd; ++i) out[i] += a * orc_f16_to_f32(vt[i]);
        }
    }
}

static void shortlist_head(OModel* m, int k, int n_valid, const int* must, int n_must);

/* head (engine/src/model.cpp:230-238). */
static void head(OModel* m, int top_k, int n_valid, const int* must, int n_must) {
    if (top_k > 0 && m->head_q4) {
        shortlist_head(m, top_k, n_valid, must, n_must);
    } else {
        linear(m, m->logits, m->lm_head, m->xq, m->xd);
        m->last_head_rows = m->lm_head->rows;
    }
}

/* Model::forward (engine/src/model.cpp:165-228), f16 KV cache.  Returns 0, or -1 on a bad position/token. */
int orc_forward(OModel* m, int token, int pos, int top_k, int n_valid, const int* must, int n_must, float* out) {
    if (pos < 0 || pos >= m->ctx || token < 0 || token >= m->embed->rows) return -1;
    const int dim = m->dim, hd = m->hd, kvd = m->n_kv * hd;
    get_row(m->x, m->embed->dtype, dim, m->embed->data, quant_bytes(m->embed), token);
    for (int l = 0; l < m->n_layers; ++l) {
        const OTensor** L = m->L + l * 12;
        rmsnorm(m->xb, m->x, (const float*)L[0]->data, dim, m->eps);
        orc_quantize_q8(m->xb, dim, m->xq, m->xd);
        linear(m, m->q, L[1], m->xq, m->xd);
        linear(m, m->k, L[2], m->xq, m->xd);
        linear(m, m->v, L[3], m->xq, m->xd);
        add_bias(m->q, L[5]);
        add_bias(m->k, L[6]);
        add_bias(m->v, L[7]);
        rope(m->q, m->n_heads, hd, pos, m->theta);
        rope(m->k, m->n_kv, hd, pos, m->theta);
        uint16_t* kc = m->kc + (size_t)l * m->ctx * kvd;
        uint16_t* vc = m->vc + (size_t)l * m->ctx * kvd;
        for (int i = 0; i < kvd; ++i) {
            kc[(size_t)pos * kvd + i] = f32_to_f16(m->k[i]);
            vc[(size_t)pos * kvd + i] = f32_to_f16(m->v[i]);
        }
        attend(m, kc, vc, pos);
        memcpy(m->dbg_q, m->q, sizeof(float) * (size_t)(m->n_heads * hd));
        memcpy(m->dbg_att, m->xb, sizeof(float) * (size_t)dim);
        orc_quantize_q8(m->xb, dim, m->xq, m->xd);
        linear(m, m->xb2, L[4], m->xq, m->xd);
        for (int i = 0; i < dim; ++i) m->x[i] += m->xb2[i];
        rmsnorm(m->xb, m->x, (const float*)L[8]->data, dim, m->eps);
        orc_quantize_q8(m->xb, dim, m->xq, m->xd);
        linear(m, m->hb, L[9], m->xq, m->xd);
        linear(m, m->hb2, L[10], m->xq, m->xd);
        for (int i = 0; i < m->ffn; ++i) { /* swiglu, engine/src/ops_ref.cpp:243-248 */
            const float g = m->hb[i];
            m->hb[i] = g / (1.0f + ref_expf(-g)) * m->hb2[i];
        }
        if (m->flags & 1u) fwht_blocks(m->hb, m->ffn, 256); /* FLAG_HADAMARD_DOWN, engine/src/model.cpp:219 */
        orc_quantize_q8(m->hb, m->ffn, m->hq, m->hd_);
        linear(m, m->xb2, L[11], m->hq, m->hd_);
        for (int i = 0; i < dim; ++i) m->x[i] += m->xb2[i];
    }
    memcpy(m->dbg_x, m->x, sizeof(float) * (size_t)dim);
    rmsnorm(m->x, m->x, (const float*)m->final_norm->data, dim, m->eps);
    orc_quantize_q8(m->x, dim, m->xq, m->xd);
    head(m, top_k, n_valid, must, n_must);
    if (out) memcpy(out, m->logits, sizeof(float) * (size_t)m->vocab);
    return 0;
}

/* Model::forward_batch (engine/src/model.cpp:349-361): bit-identical to token-by-token by construction. */
int orc_forward_batch(OModel* m, const int* tokens, int n, int pos0, int top_k, int n_valid, const int* must, int n_must,
                      float* out) {
    if (n <= 0 || pos0 < 0 || pos0 + n > m->ctx) return -1;
    for (int i = 0; i < n; ++i)
        if (orc_forward(m, tokens[i], pos0 + i, i == n - 1 ? top_k : 0, n_valid, must, n_must, i == n - 1 ? out : NULL))
            return -1;
    return 0;
}

int orc_head(OModel* m, int top_k, int n_valid, const int* must, int n_must, float* out, float* coarse, float* upper) {
    head(m, top_k, n_valid, must, n_must);
    if (out) memcpy(out, m->logits, sizeof(float) * (size_t)m->vocab);
    if (top_k > 0 && m->head_q4) {
        if (coarse) memcpy(coarse, m->coarse, sizeof(float) * (size_t)m->vocab);
        if (upper) memcpy(upper, m->upper, sizeof(float) * (size_t)m->vocab);
    }
    return m->last_head_rows;
}

/* ---------------------------------------------------------------- Exact Shortlist Head (engine/src/model.cpp:240-334) */

typedef struct {
    float v;
    int id;
} Sc;

static int by_value_desc(const void* a, const void* b) {
    const Sc *x = a, *y = b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return x->id - y->id;
}

static float exact_row(OModel* m, int r) {
    float v;
    const OTensor* W = m->lm_head;
    orc_matvec_q(W->dtype, W->rows, W->cols, W->data, m->xq, m->xd, r, r + 1, m->logits);
    v = m->logits[r];
    return v;
}

static void shortlist_head(OModel* m, int k, int n_valid, const int* must, int n_must) {
    const int V = m->lm_head->rows, nb = m->lm_head->cols / QK;
    const int nv = (n_valid > 0 && n_valid < V) ? n_valid : V;
    for (int b = 0; b < nb; ++b) { /* model.cpp:247-251 */
        float ss = 0.f;
        for (int i = 0; i < QK; ++i) ss += (float)m->xq[b * QK + i] * (float)m->xq[b * QK + i];
        m->xnorm[b] = m->xd[b] * sqrtf(ss);
    }
    for (int i = 0; i < n_must; ++i)
        if (must[i] >= 0 && must[i] < nv) m->must_mark[must[i]] = 1;
    const int n_seed = k + 8;
    orc_matvec_q(DT_Q4_0, V, m->lm_head->cols, m->head_q4->data, m->xq, m->xd, 0, V, m->coarse);
    const uint16_t* err = (const uint16_t*)m->head_err->data;
    /* seeds: the n_seed best coarse scores among valid non-must rows (model.cpp:259-284, 293-301) */
    Sc* cand = malloc(sizeof(Sc) * (size_t)V);
    int nc = 0;
    for (int r = 0; r < V; ++r) {
        float bound = 0.f;
        for (int b = 0; b < nb; ++b) bound += orc_f16_to_f32(err[(size_t)r * nb + b]) * m->xnorm[b];
        bound = bound * 1.001f + 1e-5f;
        m->upper[r] = m->coarse[r] + bound;
        m->logits[r] = -INFINITY;
        if (r >= nv || m->must_mark[r]) continue;
        cand[nc].v = m->coarse[r];
        cand[nc].id = r;
        ++nc;
    }
    qsort(cand, (size_t)nc, sizeof(Sc), by_value_desc);
    const int ns = nc < n_seed ? nc : n_seed;
    int rows = 0;
    Sc* seeds = malloc(sizeof(Sc) * (size_t)(ns > 0 ? ns : 1));
    for (int i = 0; i < ns; ++i) {
        seeds[i].id = cand[i].id;
        m->must_mark[cand[i].id] = 2;
    }
    for (int i = 0; i < ns; ++i) seeds[i].v = exact_row(m, seeds[i].id);
    rows += ns;
    float tau = -INFINITY;
    if (ns >= k) { /* model.cpp:308-313 */
        qsort(seeds, (size_t)ns, sizeof(Sc), by_value_desc);
        tau = seeds[k - 1].v;
    }
    for (int r = 0; r < nv; ++r) /* model.cpp:315-321 */
        if (!m->must_mark[r] && m->upper[r] >= tau) {
            exact_row(m, r);
            ++rows;
        }
    for (int i = 0; i < n_must; ++i) { /* model.cpp:324-330 */
        const int id = must[i];
        if (id >= 0 && id < nv && m->must_mark[id] == 1) {
            exact_row(m, id);
            ++rows;
            m->must_mark[id] = 0;
        }
    }
    for (int i = 0; i < ns; ++i) m->must_mark[seeds[i].id] = 0;
    m->last_head_rows = rows;
    free(cand);
    free(seeds);
}

/* ---------------------------------------------------------------- sampler (engine/src/sampler.cpp:22-85) */

typedef struct {
    float temperature, top_p, min_p, repeat_penalty;
    int top_k, repeat_window;
    uint64_t state;
} OSampler;

OSampler* orc_sampler_new(float temperature, int top_k, float top_p, float min_p, float repeat_penalty, int repeat_window,
                          unsigned long long seed) {
    OSampler* s = calloc(1, sizeof *s);
    s->temperature = temperature;
    s->top_k = top_k;
    s->top_p = top_p;
    s->min_p = min_p;
    s->repeat_penalty = repeat_penalty;
    s->repeat_window = repeat_window;
    s->state = (seed ? seed : 0x9E3779B97F4A7C15ULL) | 1ULL;
    return s;
}
void orc_sampler_free(OSampler* s) { free(s); }

static uint64_t next_u64(OSampler* s) { /* xorshift64*, sampler.cpp:15-20 */
    s->state ^= s->state >> 12;
    s->state ^= s->state << 25;
    s->state ^= s->state >> 27;
    return s->state * 0x2545F4914F6CDD1DULL;
}

/* Ties between equal logits go to the lower id (the reference leaves their order to nth_element/sort). */
int orc_sample(OSampler* s, float* logits, int n_valid, const int* history, int n_hist) {
    if (s->repeat_penalty != 1.0f && n_hist > 0) {
        const int from = (s->repeat_window > 0 && n_hist > s->repeat_window) ? n_hist - s->repeat_window : 0;
        uint8_t* seen = calloc((size_t)n_valid + 1, 1);
        for (int i = from; i < n_hist; ++i) {
            const int id = history[i];
            if (id < 0 || id >= n_valid || seen[id]) continue;
            seen[id] = 1;
            float* l = &logits[id];
            *l = *l > 0 ? *l / s->repeat_penalty : *l * s->repeat_penalty;
        }
        free(seen);
    }
    if (s->temperature <= 0.0f) {
        int best = 0;
        for (int i = 1; i < n_valid; ++i)
            if (logits[i] > logits[best]) best = i;
        return best;
    }
    Sc* c = malloc(sizeof(Sc) * (size_t)n_valid);
    for (int i = 0; i < n_valid; ++i) {
        c[i].v = logits[i];
        c[i].id = i;
    }
    qsort(c, (size_t)n_valid, sizeof(Sc), by_value_desc);
    int k = n_valid;
    if (s->top_k > 0 && s->top_k < k) k = s->top_k;
    const float mx = c[0].v;
    float sum = 0.f;
    for (int i = 0; i < k; ++i) {
        c[i].v = expf((c[i].v - mx) / s->temperature);
        sum += c[i].v;
    }
    for (int i = 0; i < k; ++i) c[i].v /= sum;
    int keep = k;
    if (s->min_p > 0.f) {
        const float floor_ = c[0].v * s->min_p;
        while (keep > 1 && c[keep - 1].v < floor_) --keep;
    }
    if (s->top_p < 1.f) {
        float cum = 0.f;
        for (int i = 0; i < keep; ++i) {
            cum += c[i].v;
            if (cum >= s->top_p) {
                keep = i + 1;
                break;
            }
        }
    }
    float total = 0.f;
    for (int i = 0; i < keep; ++i) total += c[i].v;
    float r = (float)(next_u64(s) >> 40) * (1.0f / 16777216.0f) * total;
    int pick = c[keep - 1].id;
    for (int i = 0; i < keep; ++i) {
        r -= c[i].v;
        if (r <= 0.f) {
            pick = c[i].id;
            break;
        }
    }
    free(c);
    return pick;
}
