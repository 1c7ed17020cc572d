/*
 * CPU ORACLE — test infrastructure only (see oracle.h).
 *
 * GGUF v3 parse (Singularity/src/core/cortex_a5_engine.cpp:429-659) and the
 * Llama decoder forward in Singularity's order
 * (Singularity/src/core/cortex_a5_engine.cpp:1029-1293), with three
 * documented departures toward llama.cpp, the engines' actual CPU path:
 * RoPE uses the θ^(−2i/hd) table for llama (adjacent pairs), K-quant weights
 * pair with Q8_K activations, and RMSNorm sums its squares in double as
 * ggml's rms_norm does (orc_rmsnorm_ggml).
 */
#include "oracle.h"

#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

typedef struct {
    int type;
    const uint8_t* data;
    int64_t ne[4];
    int n_dims;
} orc_tensor;

typedef struct {
    orc_tensor attn_norm, ffn_norm, wq, wk, wv, wo, w1, w2, w3;
} orc_layer;

struct orc_model {
    const uint8_t* base;
    size_t size;
    int mapped;
    uint8_t* owned;
    int n_layers, dim, hidden, n_heads, n_kv, vocab, ctx_len, head_dim;
    float eps, theta;
    orc_tensor embd, out_norm, out;
    orc_layer* layers;
    /* runtime */
    int n_seq, n_ctx;
    uint8_t *kc, *vc;  /* [seq][layer][pos][kv_dim], rows in the cache types' storage */
    int ktype, vtype;  /* ORC_F16 (default), ORC_Q8_0 or ORC_Q4_0 */
    float *x, *xb, *xb2, *q, *k, *v, *hb, *hb2;
    void* xq;
    float* rope;
    orc_tap_fn tap;
    void* tap_user;
    int device_order;   /* 1: evaluate in the GPU kernels' order (bit-exact check); 2: the same
                           with the projections in the reference's row order, as the
                           tensor-core prefill GEMMs compute them */
    int tp;             /* tensor-parallel ranks emulated by the row-sharded projections */
    float* part;        /* [tp][dim] partial outputs */
};

void orc_model_set_device_order(orc_model* m, int on) { m->device_order = on; }

int orc_model_set_kv_types(orc_model* m, int ktype, int vtype) {
    if ((ktype != ORC_F16 && ktype != ORC_Q8_0 && ktype != ORC_Q4_0) ||
        (vtype != ORC_F16 && vtype != ORC_Q8_0 && vtype != ORC_Q4_0))
        return -1;
    m->ktype = ktype;
    m->vtype = vtype;
    return m->kc ? orc_model_init_cache(m, m->n_seq, m->n_ctx) : 0;
}

int orc_model_set_tp(orc_model* m, int tp) {
    if (tp < 1 || m->n_heads % tp || m->n_kv % tp || m->hidden % tp || m->vocab % tp) return -1;
    /* each rank's column slice starts on an activation block (32, or 256 for K-quants) */
    const int bo = orc_vec_dot_type(m->layers[0].wo.type) == ORC_Q8_K ? 256 : 32;
    const int bd = orc_vec_dot_type(m->layers[0].w2.type) == ORC_Q8_K ? 256 : 32;
    if ((m->n_heads / tp * m->head_dim) % bo || (m->hidden / tp) % bd) return -1;
    free(m->part);
    m->part = (float*)malloc(sizeof(float) * (size_t)tp * m->dim);
    m->tp = tp;
    return m->part ? 0 : -1;
}

void orc_model_set_tap(orc_model* m, orc_tap_fn fn, void* user) {
    m->tap = fn;
    m->tap_user = user;
}
#define TAP(name, layer, ptr, n) do { if (m->tap) m->tap(name, layer, ptr, (long)(n), m->tap_user); } while (0)

static uint32_t rd_u32(const uint8_t* p) { uint32_t v; memcpy(&v, p, 4); return v; }
static uint64_t rd_u64(const uint8_t* p) { uint64_t v; memcpy(&v, p, 8); return v; }

static int key_eq(const char* k, size_t n, const char* s) { return strlen(s) == n && memcmp(k, s, n) == 0; }
static int key_ends(const char* k, size_t n, const char* s) {
    const size_t m = strlen(s);
    return n >= m && memcmp(k + n - m, s, m) == 0;
}

/* Byte size of one scalar GGUF value type; 0 for string / array. */
static size_t gguf_scalar_size(uint32_t t) {
    switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
    }
}

/* Skip one value (Milda/src/engine.cpp:89-146 skip_gguf_value, restated). */
static const uint8_t* gguf_skip(const uint8_t* p, const uint8_t* end, uint32_t t) {
    if (t == 8) {
        if (p + 8 > end) return end;
        return p + 8 + rd_u64(p);
    }
    if (t == 9) {
        if (p + 12 > end) return end;
        const uint32_t et = rd_u32(p);
        const uint64_t n = rd_u64(p + 4);
        p += 12;
        const size_t es = gguf_scalar_size(et);
        if (es) return p + es * n;
        for (uint64_t i = 0; i < n && p < end; ++i) p = gguf_skip(p, end, et);
        return p;
    }
    return p + gguf_scalar_size(t);
}

static size_t tensor_bytes(const orc_tensor* t) {
    int64_t rows = 1;
    for (int i = 1; i < t->n_dims; ++i) rows *= t->ne[i];
    return orc_row_bytes(t->type, (int)t->ne[0]) * (size_t)rows;
}

static int parse(orc_model* m) {
    const uint8_t* p = m->base;
    const uint8_t* end = m->base + m->size;
    if (m->size < 24 || rd_u32(p) != 0x46554747u) return -1;
    const uint32_t version = rd_u32(p + 4);
    if (version != 2 && version != 3) return -1;
    const uint64_t n_tensors = rd_u64(p + 8), n_kv = rd_u64(p + 16);
    p += 24;
    size_t alignment = 32;
    m->eps = 1e-5f;
    m->theta = 10000.0f;
    for (uint64_t i = 0; i < n_kv; ++i) {
        if (p + 12 > end) return -1;
        const uint64_t klen = rd_u64(p);
        const char* key = (const char*)(p + 8);
        p += 8 + klen;
        const uint32_t vt = rd_u32(p);
        p += 4;
        if (vt == 4 || vt == 5) {
            const uint32_t v = rd_u32(p);
            if (key_eq(key, klen, "general.alignment")) alignment = v;
            else if (key_ends(key, klen, ".block_count")) m->n_layers = (int)v;
            else if (key_ends(key, klen, ".embedding_length")) m->dim = (int)v;
            else if (key_ends(key, klen, ".feed_forward_length")) m->hidden = (int)v;
            else if (key_ends(key, klen, ".attention.head_count")) m->n_heads = (int)v;
            else if (key_ends(key, klen, ".attention.head_count_kv")) m->n_kv = (int)v;
            else if (key_ends(key, klen, ".context_length")) m->ctx_len = (int)v;
            else if (key_ends(key, klen, ".vocab_size")) m->vocab = (int)v;
        } else if (vt == 6) {
            float f;
            memcpy(&f, p, 4);
            if (key_ends(key, klen, ".layer_norm_rms_epsilon")) m->eps = f;
            else if (key_ends(key, klen, ".rope.freq_base")) m->theta = f;
        }
        p = gguf_skip(p, end, vt);
        if (p > end) return -1;
    }
    if (m->n_layers <= 0 || m->dim <= 0 || (m->dim & 31) || m->n_heads <= 0) return -1;
    if (m->n_kv <= 0) m->n_kv = m->n_heads;
    m->layers = (orc_layer*)calloc((size_t)m->n_layers, sizeof(orc_layer));
    orc_tensor* tab = (orc_tensor*)calloc(n_tensors ? n_tensors : 1, sizeof(orc_tensor));
    char** names = (char**)calloc(n_tensors ? n_tensors : 1, sizeof(char*));
    size_t* offs = (size_t*)calloc(n_tensors ? n_tensors : 1, sizeof(size_t));
    for (uint64_t i = 0; i < n_tensors; ++i) {
        if (p + 8 > end) return -1;
        const uint64_t nlen = rd_u64(p);
        names[i] = (char*)calloc(nlen + 1, 1);
        memcpy(names[i], p + 8, nlen);
        p += 8 + nlen;
        const uint32_t nd = rd_u32(p);
        p += 4;
        tab[i].n_dims = (int)nd;
        for (uint32_t d = 0; d < 4; ++d) tab[i].ne[d] = 1;
        for (uint32_t d = 0; d < nd; ++d) {
            if (d < 4) tab[i].ne[d] = (int64_t)rd_u64(p);
            p += 8;
        }
        tab[i].type = (int)rd_u32(p);
        offs[i] = (size_t)rd_u64(p + 4);
        p += 12;
    }
    const size_t hdr = (size_t)(p - m->base);
    const size_t data_off = (hdr + alignment - 1) / alignment * alignment;
    for (uint64_t i = 0; i < n_tensors; ++i) {
        orc_tensor t = tab[i];
        t.data = m->base + data_off + offs[i];
        if (t.data + tensor_bytes(&t) > end) return -1;
        const char* n = names[i];
        if (!strcmp(n, "token_embd.weight")) m->embd = t;
        else if (!strcmp(n, "output_norm.weight")) m->out_norm = t;
        else if (!strcmp(n, "output.weight")) m->out = t;
        else if (!strncmp(n, "blk.", 4)) {
            char* e;
            const long l = strtol(n + 4, &e, 10);
            if (l >= 0 && l < m->n_layers && *e == '.') {
                orc_layer* L = &m->layers[l];
                const char* s = e + 1;
                if (!strcmp(s, "attn_norm.weight")) L->attn_norm = t;
                else if (!strcmp(s, "ffn_norm.weight")) L->ffn_norm = t;
                else if (!strcmp(s, "attn_q.weight")) L->wq = t;
                else if (!strcmp(s, "attn_k.weight")) L->wk = t;
                else if (!strcmp(s, "attn_v.weight")) L->wv = t;
                else if (!strcmp(s, "attn_output.weight")) L->wo = t;
                else if (!strcmp(s, "ffn_gate.weight")) L->w1 = t;
                else if (!strcmp(s, "ffn_down.weight")) L->w2 = t;
                else if (!strcmp(s, "ffn_up.weight")) L->w3 = t;
            }
        }
        free(names[i]);
    }
    free(names);
    free(offs);
    free(tab);
    if (!m->embd.data || !m->out_norm.data) return -1;
    if (!m->out.data) m->out = m->embd; /* tied head, Singularity :650-654 */
    if (m->vocab <= 0) m->vocab = (int)m->out.ne[1];
    if (m->hidden <= 0 && m->layers[0].w1.data) m->hidden = (int)m->layers[0].w1.ne[1];
    m->head_dim = m->dim / m->n_heads;
    for (int l = 0; l < m->n_layers; ++l) {
        const orc_layer* L = &m->layers[l];
        if (!L->attn_norm.data || !L->ffn_norm.data || !L->wq.data || !L->wk.data || !L->wv.data ||
            !L->wo.data || !L->w1.data || !L->w2.data || !L->w3.data)
            return -1;
    }
    return 0;
}

orc_model* orc_model_from_memory(const void* data, size_t size) {
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->ktype = m->vtype = ORC_F16;
    m->base = (const uint8_t*)data;
    m->size = size;
    if (parse(m) != 0) {
        orc_model_free(m);
        return NULL;
    }
    return m;
}

orc_model* orc_model_open(const char* path) {
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return NULL;
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); return NULL; }
    void* p = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return NULL;
    orc_model* m = orc_model_from_memory(p, (size_t)st.st_size);
    if (!m) { munmap(p, (size_t)st.st_size); return NULL; }
    m->mapped = 1;
    return m;
}

void orc_model_free(orc_model* m) {
    if (!m) return;
    if (m->mapped) munmap((void*)m->base, m->size);
    free(m->layers);
    free(m->kc); free(m->vc);
    free(m->x); free(m->xb); free(m->xb2); free(m->q); free(m->k); free(m->v);
    free(m->hb); free(m->hb2); free(m->xq); free(m->rope); free(m->part);
    free(m);
}

int orc_model_info(const orc_model* m, int32_t* out, int n) {
    const int32_t v[12] = {m->n_layers, m->dim, m->hidden, m->n_heads, m->n_kv, m->vocab,
                           m->head_dim, m->ctx_len, m->layers[0].wq.type, m->embd.type, m->out.type,
                           (int32_t)0};
    for (int i = 0; i < n && i < 12; ++i) out[i] = v[i];
    return 12;
}

int orc_model_init_cache(orc_model* m, int n_seq, int n_ctx) {
    const int kv_dim = m->head_dim * m->n_kv;
    free(m->kc); free(m->vc); free(m->rope);
    m->n_seq = n_seq;
    m->n_ctx = n_ctx;
    const size_t n = (size_t)n_seq * m->n_layers * n_ctx;
    m->kc = (uint8_t*)calloc(n, orc_row_bytes(m->ktype, kv_dim));
    m->vc = (uint8_t*)calloc(n, orc_row_bytes(m->vtype, kv_dim));
    m->rope = (float*)malloc(sizeof(float) * (size_t)n_ctx * m->head_dim);
    orc_rope_table(m->theta, m->head_dim, 0, n_ctx, m->rope);
    const int big = m->dim > m->hidden ? m->dim : m->hidden;
    if (!m->x) {
        m->x = (float*)calloc((size_t)m->dim, 4);
        m->xb = (float*)calloc((size_t)big, 4);
        m->xb2 = (float*)calloc((size_t)big, 4);
        m->q = (float*)calloc((size_t)m->dim, 4);
        m->k = (float*)calloc((size_t)kv_dim, 4);
        m->v = (float*)calloc((size_t)kv_dim, 4);
        m->hb = (float*)calloc((size_t)m->hidden, 4);
        m->hb2 = (float*)calloc((size_t)m->hidden, 4);
        m->xq = calloc((size_t)big / 32 + 8, ORC_Q8_K_BYTES);
    }
    return (m->kc && m->vc) ? 0 : -1;
}

/* fp16 rows take `bits` in every value; Q8_0 rows take `bits` as every
 * block's scale and 1 as every code. */
static void cache_fill_rows(uint8_t* c, int type, size_t n_vals, uint16_t bits) {
    if (type == ORC_Q4_0) {
        for (size_t b = 0; b < n_vals / 32; ++b) {
            uint8_t* blk = c + b * ORC_Q4_0_BYTES;
            memcpy(blk, &bits, 2);
            memset(blk + 2, 0x99, 16);
        }
    } else if (type == ORC_Q8_0) {
        for (size_t b = 0; b < n_vals / 32; ++b) {
            uint8_t* blk = c + b * ORC_Q8_0_BYTES;
            memcpy(blk, &bits, 2);
            memset(blk + 2, 1, 32);
        }
    } else {
        for (size_t i = 0; i < n_vals; ++i) memcpy(c + 2 * i, &bits, 2);
    }
}

void orc_model_cache_fill(orc_model* m, uint16_t bits) {
    const size_t n = (size_t)m->n_seq * m->n_layers * m->n_ctx * m->head_dim * m->n_kv;
    cache_fill_rows(m->kc, m->ktype, n, bits);
    cache_fill_rows(m->vc, m->vtype, n, bits);
}

/* matmul_quantized with the activation quantized for the weight's dot type
 * (Singularity quantizes to Q8_0 before every projection, :1127, :1257,
 * :1269, :1275, :1290; K-quant weights take Q8_K as in ggml). */
static void proj_mode(orc_model* m, const orc_tensor* w, const float* x, float* y, int nt, int swiglu) {
    const int k = (int)w->ne[0];
    if (orc_vec_dot_type(w->type) == ORC_Q8_K) orc_quantize_row_q8_k(x, m->xq, k);
    else orc_quantize_row_q8_0(x, m->xq, k);
    if (m->device_order == 1) orc_matmul_dev(w->type, w->data, w->ne[1], k, m->xq, y, swiglu, nt);
    else orc_matmul(w->type, w->data, w->ne[1], k, m->xq, y, nt);
}
static void proj(orc_model* m, const orc_tensor* w, const float* x, float* y, int nt) { proj_mode(m, w, x, y, nt, 0); }

/* Attention-out and FFN-down under tensor parallelism: rank r owns input
 * columns [r*k/tp, (r+1)*k/tp) and produces a partial output over them (in
 * the reference's order over its blocks, or the tile order of device-order
 * mode); the partials are summed in rank order, y = ((p0 + p1) + p2) + ...,
 * which is the reduction the GPU ranks perform after exchanging partials. */
static void proj_reduce(orc_model* m, const orc_tensor* w, const float* x, float* y, int nt) {
    if (m->tp <= 1 || m->device_order == 2) { proj(m, w, x, y, nt); return; }
    const int k = (int)w->ne[0], n = (int)w->ne[1], kl = k / m->tp;
    const int at = orc_vec_dot_type(w->type);
    if (at == ORC_Q8_K) orc_quantize_row_q8_k(x, m->xq, k);
    else orc_quantize_row_q8_0(x, m->xq, k);
    const size_t rb = orc_row_bytes(w->type, k);
    for (int r = 0; r < m->tp; ++r) {
        const uint8_t* ws = w->data + orc_row_bytes(w->type, r * kl);
        const void* xs = (const uint8_t*)m->xq + orc_row_bytes(at, r * kl);
        if (m->device_order == 1) orc_matmul_dev_strided(w->type, ws, n, rb, kl, xs, m->part + (size_t)r * n, 0, nt);
        else orc_matmul_strided(w->type, ws, n, rb, kl, xs, m->part + (size_t)r * n, nt);
    }
    for (int i = 0; i < n; ++i) {
        float s = m->part[i];
        for (int r = 1; r < m->tp; ++r) s = s + m->part[(size_t)r * n + i];
        y[i] = s;
    }
}

int orc_model_forward_range(orc_model* m, int seq, int32_t token, int pos, int l0, int l1, float* logits,
                            int nt) {
    if (!m->kc || seq < 0 || seq >= m->n_seq || pos < 0 || pos >= m->n_ctx) return -1;
    if (token < 0 || token >= (int32_t)m->embd.ne[1]) token = 0;
    const int dim = m->dim, hd = m->head_dim, nkv = m->n_kv, kv_dim = hd * nkv;
    if (l0 <= 0) {
        /* 1. embedding row (:1066-1105) */
        orc_dequantize_row(m->embd.type, m->embd.data + orc_row_bytes(m->embd.type, dim) * (size_t)token,
                           m->x, dim);
        TAP("embed", -1, m->x, dim);
        l0 = 0;
    }
    const float* cs = m->rope + (size_t)pos * hd;
    const size_t krb = orc_row_bytes(m->ktype, kv_dim), vrb = orc_row_bytes(m->vtype, kv_dim);
    const int typed = m->ktype != ORC_F16 || m->vtype != ORC_F16;
    const int nl = l1 < m->n_layers ? l1 : m->n_layers;
    for (int l = l0; l < nl; ++l) {
        const orc_layer* L = &m->layers[l];
        orc_rmsnorm_ggml(m->x, (const float*)L->attn_norm.data, m->xb, dim, m->eps); /* :1121 */
        TAP("attn_norm", l, m->xb, dim);
        proj(m, &L->wq, m->xb, m->q, nt);                                             /* :1129 */
        proj(m, &L->wk, m->xb, m->k, nt);
        proj(m, &L->wv, m->xb, m->v, nt);
        TAP("q", l, m->q, dim);
        TAP("k", l, m->k, kv_dim);
        TAP("v", l, m->v, kv_dim);
        orc_rope_pairs(m->q, cs, hd, m->n_heads);                                     /* :1187 */
        orc_rope_pairs(m->k, cs, hd, nkv);
        TAP("q_rope", l, m->q, dim);
        const size_t cache_row = ((size_t)seq * m->n_layers + l) * m->n_ctx;
        uint8_t* kc = m->kc + cache_row * krb;
        uint8_t* vc = m->vc + cache_row * vrb;
        orc_kv_store_row(m->ktype, m->k, kc + (size_t)pos * krb, kv_dim);             /* :1195 */
        orc_kv_store_row(m->vtype, m->v, vc + (size_t)pos * vrb, kv_dim);
        if (typed)
            orc_attn_decode_typed(m->q, kc, m->ktype, krb, vc, m->vtype, vrb, pos + 1, m->n_heads, nkv, hd, m->xb);
        else if (m->device_order)
            orc_attn_decode_dev(m->q, (const uint16_t*)kc, (const uint16_t*)vc, kv_dim, pos + 1, m->n_heads, nkv,
                                hd, m->xb);
        else
            orc_attn_decode(m->q, (const uint16_t*)kc, (const uint16_t*)vc, kv_dim, pos + 1, m->n_heads, nkv, hd,
                            m->xb);                                                   /* :1205 */
        TAP("attn_out", l, m->xb, dim);
        proj_reduce(m, &L->wo, m->xb, m->xb2, nt);                                    /* :1256 */
        TAP("attn_proj", l, m->xb2, dim);
        for (int i = 0; i < dim; ++i) m->x[i] += m->xb2[i];
        orc_rmsnorm_ggml(m->x, (const float*)L->ffn_norm.data, m->xb, dim, m->eps);  /* :1264 */
        TAP("ffn_norm", l, m->xb, dim);
        proj_mode(m, &L->w1, m->xb, m->hb, nt, 1);                                    /* :1270 */
        proj_mode(m, &L->w3, m->xb, m->hb2, nt, 1);
        if (m->device_order) orc_silu_mul_dev(m->hb, m->hb2, m->hidden);
        else orc_silu_mul(m->hb, m->hb2, m->hidden);                                  /* :1277 */
        TAP("ffn_act", l, m->hb, m->hidden);
        proj_reduce(m, &L->w2, m->hb, m->xb, nt);                                     /* :1280 */
        TAP("ffn_out", l, m->xb, dim);
        for (int i = 0; i < dim; ++i) m->x[i] += m->xb[i];
    }
    if (!logits) return 0;
    orc_rmsnorm_ggml(m->x, (const float*)m->out_norm.data, m->xb, dim, m->eps);      /* :1287 */
    TAP("result_norm", -1, m->xb, dim);
    proj(m, &m->out, m->xb, logits, nt);                                              /* :1292 */
    return 0;
}

int orc_model_forward_layers(orc_model* m, int seq, int32_t token, int pos, float* logits, int nt,
                             int n_layers_run) {
    return orc_model_forward_range(m, seq, token, pos, 0, n_layers_run, logits, nt);
}

int orc_model_forward(orc_model* m, int seq, int32_t token, int pos, float* logits, int nt) {
    return orc_model_forward_layers(m, seq, token, pos, logits, nt, m->n_layers);
}

int orc_model_hidden(const orc_model* m, float* out, int n) {
    for (int i = 0; i < n && i < m->dim; ++i) out[i] = m->x[i];
    return m->dim;
}

/* Milda shift_kv_cache_in_place (Milda/src/engine.cpp:1642-1675) on one
 * sequence: drop positions [p0, p1), move [p1, n_past) down to p0 and
 * re-rotate those K rows by −(p1−p0). */
int orc_model_kv_shift(orc_model* m, int seq, int p0, int p1, int n_past) {
    if (!m->kc || p0 < 0 || p1 < p0 || n_past < p1 || n_past > m->n_ctx) return -1;
    const int kv_dim = m->head_dim * m->n_kv;
    const size_t krb = orc_row_bytes(m->ktype, kv_dim), vrb = orc_row_bytes(m->vtype, kv_dim);
    const int n_move = n_past - p1;
    for (int l = 0; l < m->n_layers; ++l) {
        const size_t cache_row = ((size_t)seq * m->n_layers + l) * m->n_ctx;
        uint8_t* kc = m->kc + cache_row * krb;
        uint8_t* vc = m->vc + cache_row * vrb;
        memmove(kc + (size_t)p0 * krb, kc + (size_t)p1 * krb, (size_t)n_move * krb);
        memmove(vc + (size_t)p0 * vrb, vc + (size_t)p1 * vrb, (size_t)n_move * vrb);
        if (m->ktype == ORC_F16)
            orc_kv_shift_k((uint16_t*)(kc + (size_t)p0 * krb), kv_dim, n_move, m->n_kv, m->head_dim, -(p1 - p0),
                           m->theta);
        else
            orc_kv_shift_k_typed(kc + (size_t)p0 * krb, m->ktype, krb, n_move, m->n_kv, m->head_dim, -(p1 - p0),
                                 m->theta);
    }
    return 0;
}
