/*
 * tos_gguf.c - GGUF container (v2 / v3) reader and the llama-family tensor
 * mapping onto tos_model_desc_t (runtime/nn/gguf.c:204-423 parse and
 * lookups, runtime/nn/llm.c:1374-1448 tensor names, llm.c:1521-1545
 * architecture parameters).
 *
 * The file is parsed in place: tensor data pointers point into the caller's
 * buffer (or into a read-only mapping made by tos_gguf_open_file), so a
 * model descriptor built from it uploads the GGUF blocks directly.  Every
 * read is bounds-checked; malformed input returns TOS_EINVAL.
 *
 * Differences from the reference, on purpose:
 *  - without "<arch>.vocab_size" the vocabulary is token_embd's second
 *    dimension (its row count; the reference reads the first, the row
 *    length);
 *  - F16 norm weights are widened into buffers owned by the reader (the
 *    device model takes F32 norms);
 *  - limits are the file's own (no fixed tables of 512 keys / 4096 tensors).
 */
#include <fcntl.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "tos_internal.h"

#define GGUF_MAGIC 0x46554747u   /* "GGUF" little-endian */

enum {
    GT_U8 = 0, GT_I8 = 1, GT_U16 = 2, GT_I16 = 3, GT_U32 = 4, GT_I32 = 5, GT_F32 = 6, GT_BOOL = 7,
    GT_STRING = 8, GT_ARRAY = 9, GT_U64 = 10, GT_I64 = 11, GT_F64 = 12
};

typedef struct {
    const char *p;      /* not NUL-terminated: points into the file */
    uint64_t len;
} gstr_t;

typedef struct {
    gstr_t key;
    uint32_t type;
    uint64_t u;         /* integer / bool value (zero- or sign-extended) */
    double f;           /* float value */
    gstr_t s;           /* string value */
    uint32_t arr_type;  /* array element type */
    uint64_t arr_n;
} gkv_t;

typedef struct {
    char *name;         /* NUL-terminated copy */
    uint32_t n_dims;
    uint64_t dims[4];
    uint32_t type;
    uint64_t offset;
    uint64_t bytes;
    const void *data;
} gtensor_t;

struct tos_gguf {
    const uint8_t *base;
    uint64_t size;
    void *map;          /* mmap'd file (tos_gguf_open_file) */
    uint32_t version;
    gkv_t *kv;
    uint64_t n_kv;
    gtensor_t *t;
    uint64_t n_t;
    /* storage handed out through tos_gguf_model_desc */
    const void **ptrs;  /* 9 arrays of n_layers pointers */
    float *norm_f32;    /* widened F16 norms */
};

typedef struct {
    const uint8_t *p;
    uint64_t n, pos;
    int bad;
} rd_t;

static int rd_has(rd_t *r, uint64_t n)
{
    if (r->bad || n > r->n - r->pos) {
        r->bad = 1;
        return 0;
    }
    return 1;
}

static uint64_t rd_le(rd_t *r, int bytes)
{
    if (!rd_has(r, (uint64_t)bytes)) return 0;
    uint64_t v = 0;
    for (int i = 0; i < bytes; i++) v |= (uint64_t)r->p[r->pos + i] << (8 * i);
    r->pos += (uint64_t)bytes;
    return v;
}

static gstr_t rd_str(rd_t *r)
{
    gstr_t s = {NULL, 0};
    uint64_t len = rd_le(r, 8);
    if (!rd_has(r, len)) return s;
    s.p = (const char *)r->p + r->pos;
    s.len = len;
    r->pos += len;
    return s;
}

static int scalar_size(uint32_t t)
{
    switch (t) {
    case GT_U8: case GT_I8: case GT_BOOL: return 1;
    case GT_U16: case GT_I16: return 2;
    case GT_U32: case GT_I32: case GT_F32: return 4;
    case GT_U64: case GT_I64: case GT_F64: return 8;
    default: return 0;
    }
}

static void rd_scalar(rd_t *r, uint32_t t, gkv_t *kv)
{
    const int n = scalar_size(t);
    uint64_t v = rd_le(r, n);
    kv->u = v;
    switch (t) {
    case GT_I8: kv->u = (uint64_t)(int64_t)(int8_t)v; break;
    case GT_I16: kv->u = (uint64_t)(int64_t)(int16_t)v; break;
    case GT_I32: kv->u = (uint64_t)(int64_t)(int32_t)v; break;
    case GT_F32: { uint32_t b = (uint32_t)v; float f; memcpy(&f, &b, 4); kv->f = f; break; }
    case GT_F64: { double d; memcpy(&d, &v, 8); kv->f = d; break; }
    default: break;
    }
}

/* Bytes of n elements of a ggml tensor type (ggml block sizes), 0 when the
 * type is unknown or n is not a whole number of blocks. */
static uint64_t type_bytes(uint32_t type, uint64_t n)
{
    uint64_t blk, bytes;
    switch (type) {
    case 0: blk = 1; bytes = 4; break;          /* F32 */
    case 1: blk = 1; bytes = 2; break;          /* F16 */
    case 2: blk = 32; bytes = 18; break;        /* Q4_0 */
    case 3: blk = 32; bytes = 20; break;        /* Q4_1 */
    case 6: blk = 32; bytes = 22; break;        /* Q5_0 */
    case 7: blk = 32; bytes = 24; break;        /* Q5_1 */
    case 8: blk = 32; bytes = 34; break;        /* Q8_0 */
    case 9: blk = 32; bytes = 36; break;        /* Q8_1 */
    case 10: blk = 256; bytes = 84; break;      /* Q2_K */
    case 11: blk = 256; bytes = 110; break;     /* Q3_K */
    case 12: blk = 256; bytes = 144; break;     /* Q4_K */
    case 13: blk = 256; bytes = 176; break;     /* Q5_K */
    case 14: blk = 256; bytes = 210; break;     /* Q6_K */
    default: return 0;
    }
    if (n % blk) return 0;
    if (n / blk > UINT64_MAX / bytes) return 0;   /* the byte size would wrap */
    return n / blk * bytes;
}

/* A mapped tensor has the shape the model reads from it: ne0 x ne1 elements
 * (GGUF order, ne0 fastest), every further dimension 1, a known type, and
 * data inside the file (its byte size, from the shape, was range-checked at
 * open).  Without this a tensor smaller than the header implies would pass
 * the container check and the model upload would read past it. */
static int tensor_is(const gtensor_t *t, uint64_t ne0, uint64_t ne1)
{
    if (!t->data || t->bytes == 0 || t->dims[0] != ne0) return 0;
    for (uint32_t d = 1; d < t->n_dims; d++)
        if (t->dims[d] != (d == 1 ? ne1 : 1)) return 0;
    if (t->n_dims < 2 && ne1 != 1) return 0;
    return t->bytes == type_bytes(t->type, ne0 * ne1);
}

static int gstr_eq(gstr_t s, const char *c)
{
    size_t n = strlen(c);
    return s.len == n && memcmp(s.p, c, n) == 0;
}

void tos_gguf_close(tos_gguf_t *g)
{
    if (!g) return;
    for (uint64_t i = 0; g->t && i < g->n_t; i++) free(g->t[i].name);
    free(g->t);
    free(g->kv);
    free(g->ptrs);
    free(g->norm_f32);
    if (g->map) munmap(g->map, (size_t)g->size);
    free(g);
}

int tos_gguf_open(tos_gguf_t **out, const void *data, uint64_t size)
{
    if (!out) return tos_set_status(TOS_EINVAL);
    *out = NULL;
    if (!data || size < 24) return tos_set_status(TOS_EINVAL);
    tos_gguf_t *g = (tos_gguf_t *)calloc(1, sizeof(*g));
    if (!g) return tos_set_status(TOS_ENOMEM);
    g->base = (const uint8_t *)data;
    g->size = size;
    rd_t r = {g->base, size, 0, 0};
    int rc = TOS_EINVAL;
    if (rd_le(&r, 4) != GGUF_MAGIC) goto fail;
    g->version = (uint32_t)rd_le(&r, 4);
    if (g->version < 2 || g->version > 3) { rc = TOS_ENOTSUP; goto fail; }
    g->n_t = rd_le(&r, 8);
    g->n_kv = rd_le(&r, 8);
    /* every key and tensor takes at least 8+ bytes: counts beyond the file
     * size are malformed (and would overflow the allocations) */
    if (r.bad || g->n_t > size / 8 || g->n_kv > size / 8) goto fail;
    g->kv = (gkv_t *)calloc(g->n_kv ? g->n_kv : 1, sizeof(gkv_t));
    g->t = (gtensor_t *)calloc(g->n_t ? g->n_t : 1, sizeof(gtensor_t));
    if (!g->kv || !g->t) { rc = TOS_ENOMEM; goto fail; }
    for (uint64_t i = 0; i < g->n_kv && !r.bad; i++) {
        gkv_t *kv = &g->kv[i];
        kv->key = rd_str(&r);
        kv->type = (uint32_t)rd_le(&r, 4);
        if (kv->type == GT_STRING) {
            kv->s = rd_str(&r);
        } else if (kv->type == GT_ARRAY) {
            kv->arr_type = (uint32_t)rd_le(&r, 4);
            kv->arr_n = rd_le(&r, 8);
            if (kv->arr_type == GT_STRING) {
                for (uint64_t j = 0; j < kv->arr_n && !r.bad; j++) (void)rd_str(&r);
            } else {
                const int es = scalar_size(kv->arr_type);
                if (!es || kv->arr_n > (r.n - r.pos) / (uint64_t)es) { r.bad = 1; break; }
                r.pos += kv->arr_n * (uint64_t)es;
            }
        } else if (scalar_size(kv->type)) {
            rd_scalar(&r, kv->type, kv);
        } else {
            r.bad = 1;
        }
    }
    for (uint64_t i = 0; i < g->n_t && !r.bad; i++) {
        gtensor_t *t = &g->t[i];
        gstr_t nm = rd_str(&r);
        t->n_dims = (uint32_t)rd_le(&r, 4);
        if (r.bad || t->n_dims < 1 || t->n_dims > 4) { r.bad = 1; break; }
        uint64_t n = 1;
        for (uint32_t d = 0; d < t->n_dims; d++) {
            t->dims[d] = rd_le(&r, 8);
            if (t->dims[d] == 0 || n > UINT64_MAX / t->dims[d]) r.bad = 1;
            else n *= t->dims[d];
        }
        t->type = (uint32_t)rd_le(&r, 4);
        t->offset = rd_le(&r, 8);
        t->bytes = type_bytes(t->type, n);
        t->name = (char *)malloc(nm.len + 1);
        if (!t->name) { rc = TOS_ENOMEM; goto fail; }
        if (nm.len) memcpy(t->name, nm.p, nm.len);
        t->name[nm.len] = 0;
    }
    if (r.bad) goto fail;
    /* data section: after the tensor infos, aligned (general.alignment,
     * default 32; gguf.c:294-301) */
    uint64_t align = 32;
    for (uint64_t i = 0; i < g->n_kv; i++)
        if (gstr_eq(g->kv[i].key, "general.alignment") && g->kv[i].type == GT_U32 && g->kv[i].u)
            align = g->kv[i].u;
    uint64_t data_off = (r.pos + align - 1) / align * align;
    if (data_off > size) goto fail;
    for (uint64_t i = 0; i < g->n_t; i++) {
        gtensor_t *t = &g->t[i];
        if (t->bytes) {
            if (t->offset > size - data_off || t->bytes > size - data_off - t->offset) goto fail;
            t->data = g->base + data_off + t->offset;
        }
    }
    *out = g;
    return tos_set_status(TOS_OK);
fail:
    tos_gguf_close(g);
    return tos_set_status(rc);
}

int tos_gguf_open_file(tos_gguf_t **out, const char *path)
{
    if (!out || !path) return tos_set_status(TOS_EINVAL);
    *out = NULL;
    int fd = open(path, O_RDONLY);
    if (fd < 0) return tos_set_status(TOS_EINVAL);
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size <= 0) {
        close(fd);
        return tos_set_status(TOS_EINVAL);
    }
    void *map = mmap(NULL, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return tos_set_status(TOS_ENOMEM);
    int rc = tos_gguf_open(out, map, (uint64_t)sb.st_size);
    if (rc) {
        munmap(map, (size_t)sb.st_size);
        return rc;
    }
    (*out)->map = map;
    return TOS_OK;
}

uint32_t tos_gguf_version(const tos_gguf_t *g) { return g ? g->version : 0; }
int64_t tos_gguf_n_tensors(const tos_gguf_t *g) { return g ? (int64_t)g->n_t : -1; }
int64_t tos_gguf_n_kv(const tos_gguf_t *g) { return g ? (int64_t)g->n_kv : -1; }

int64_t tos_gguf_find_tensor(const tos_gguf_t *g, const char *name)
{
    if (!g || !name) return -1;
    for (uint64_t i = 0; i < g->n_t; i++)
        if (strcmp(g->t[i].name, name) == 0) return (int64_t)i;
    return -1;
}

int tos_gguf_tensor_info(const tos_gguf_t *g, int64_t i, const char **name, int *type, int *n_dims,
                         uint64_t dims[4], const void **data, uint64_t *bytes)
{
    if (!g || i < 0 || (uint64_t)i >= g->n_t) return tos_set_status(TOS_EINVAL);
    const gtensor_t *t = &g->t[i];
    if (name) *name = t->name;
    if (type) *type = (int)t->type;
    if (n_dims) *n_dims = (int)t->n_dims;
    if (dims)
        for (int d = 0; d < 4; d++) dims[d] = d < (int)t->n_dims ? t->dims[d] : 1;
    if (data) *data = t->data;
    if (bytes) *bytes = t->bytes;
    return tos_set_status(TOS_OK);
}

static const gkv_t *find_kv(const tos_gguf_t *g, const char *key)
{
    for (uint64_t i = 0; g && key && i < g->n_kv; i++)
        if (gstr_eq(g->kv[i].key, key)) return &g->kv[i];
    return NULL;
}

/* gguf.c:392-403: any integer type is accepted for a u32 query */
int tos_gguf_get_u32(const tos_gguf_t *g, const char *key, uint32_t *out)
{
    const gkv_t *kv = find_kv(g, key);
    if (!kv || !out) return tos_set_status(TOS_EINVAL);
    switch (kv->type) {
    case GT_U8: case GT_I8: case GT_U16: case GT_I16: case GT_U32: case GT_I32: case GT_U64: case GT_I64:
        *out = (uint32_t)kv->u;
        return tos_set_status(TOS_OK);
    default:
        return tos_set_status(TOS_EINVAL);
    }
}

int tos_gguf_get_f32(const tos_gguf_t *g, const char *key, float *out)
{
    const gkv_t *kv = find_kv(g, key);
    if (!kv || !out) return tos_set_status(TOS_EINVAL);
    if (kv->type == GT_F32 || kv->type == GT_F64) {
        *out = (float)kv->f;
        return tos_set_status(TOS_OK);
    }
    return tos_set_status(TOS_EINVAL);
}

int tos_gguf_get_str(const tos_gguf_t *g, const char *key, const char **str, uint64_t *len)
{
    const gkv_t *kv = find_kv(g, key);
    if (!kv || kv->type != GT_STRING || !str || !len) return tos_set_status(TOS_EINVAL);
    *str = kv->s.p;
    *len = kv->s.len;
    return tos_set_status(TOS_OK);
}

static uint32_t get_u32_or(const tos_gguf_t *g, const char *key, uint32_t dflt)
{
    uint32_t v;
    return tos_gguf_get_u32(g, key, &v) == TOS_OK ? v : dflt;
}

static float fp16_to_f32(uint16_t h)
{
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1F, m = h & 0x3FF;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = s;
        } else {   /* subnormal: renormalise */
            uint32_t mm = m, ee = 113;
            while (!(mm & 0x400)) { mm <<= 1; ee--; }
            bits = s | (ee << 23) | ((mm & 0x3FF) << 13);
        }
    } else if (e == 31) {
        bits = s | 0x7F800000u | (m << 13);
    } else {
        bits = s | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* llama-family mapping (llm.c:1374-1448, 1521-1545).  Fills the
 * architecture and the tensor pointers of d; d->max_seq, kv_type and the
 * arithmetic modes are left to the caller (max_seq defaults to the file's
 * context length). */
int tos_gguf_model_desc(tos_gguf_t *g, tos_model_desc_t *d)
{
    if (!g || !d) return tos_set_status(TOS_EINVAL);
    char arch[64] = "llama";
    const char *as;
    uint64_t al;
    if (tos_gguf_get_str(g, "general.architecture", &as, &al) == TOS_OK) {
        if (al >= sizeof(arch)) return tos_set_status(TOS_ENOTSUP);
        memcpy(arch, as, al);
        arch[al] = 0;
    }
    char key[128];
#define AKEY(s) (snprintf(key, sizeof(key), "%s." s, arch), key)
    memset(d, 0, sizeof(*d));
    d->dim = (int)get_u32_or(g, AKEY("embedding_length"), 0);
    d->n_layers = (int)get_u32_or(g, AKEY("block_count"), 0);
    d->n_heads = (int)get_u32_or(g, AKEY("attention.head_count"), 0);
    d->n_kv_heads = (int)get_u32_or(g, AKEY("attention.head_count_kv"), (uint32_t)d->n_heads);
    d->ff_dim = (int)get_u32_or(g, AKEY("feed_forward_length"), 0);
    d->max_seq = (int)get_u32_or(g, AKEY("context_length"), 2048);
    d->vocab_size = (int)get_u32_or(g, AKEY("vocab_size"), 0);
    float f;
    d->rope_base = tos_gguf_get_f32(g, AKEY("rope.freq_base"), &f) == TOS_OK && f >= 1.0f ? f : 10000.0f;
    d->norm_eps = tos_gguf_get_f32(g, AKEY("attention.layer_norm_rms_epsilon"), &f) == TOS_OK ? f : 1e-6f;
#undef AKEY
    tos_set_status(TOS_OK);
    if (d->dim <= 0 || d->n_layers <= 0 || d->n_heads <= 0 || d->ff_dim <= 0) return tos_set_status(TOS_EINVAL);
    if (d->n_kv_heads <= 0) d->n_kv_heads = d->n_heads;
    if (d->dim % d->n_heads || d->n_heads % d->n_kv_heads) return tos_set_status(TOS_EINVAL);
    /* rows of each projection (llm.c:1541: head_dim = dim / n_heads) */
    const uint64_t dim = (uint64_t)d->dim, ff = (uint64_t)d->ff_dim;
    const uint64_t q_rows = dim, kv_rows = (uint64_t)d->n_kv_heads * (dim / (uint64_t)d->n_heads);

    int64_t ie = tos_gguf_find_tensor(g, "token_embd.weight");
    int64_t io = tos_gguf_find_tensor(g, "output_norm.weight");
    if (ie < 0 || io < 0 || !g->t[ie].data || !g->t[io].data) return tos_set_status(TOS_EINVAL);
    const gtensor_t *te = &g->t[ie];
    if (d->vocab_size <= 0) d->vocab_size = te->n_dims >= 2 && te->dims[1] <= INT32_MAX ? (int)te->dims[1] : 0;
    /* a vocab_size key must match the embedding's rows: the model uploads
     * vocab_size rows of it */
    if (d->vocab_size <= 0 || !tensor_is(te, dim, (uint64_t)d->vocab_size)) return tos_set_status(TOS_EINVAL);
    if (!tensor_is(&g->t[io], dim, 1)) return tos_set_status(TOS_EINVAL);
    d->token_embd = te->data;
    d->embd_type = (int)te->type;
    int64_t ih = tos_gguf_find_tensor(g, "output.weight");
    if (ih >= 0 && g->t[ih].data) {
        if (!tensor_is(&g->t[ih], dim, (uint64_t)d->vocab_size)) return tos_set_status(TOS_EINVAL);
        d->output_weight = g->t[ih].data;
        d->out_type = (int)g->t[ih].type;
    } else {
        d->output_weight = NULL;   /* tied to the embeddings (llm.c:1397-1407) */
        d->out_type = d->embd_type;
    }

    static const char *const suffix[9] = {"attn_norm.weight", "ffn_norm.weight", "attn_q.weight",
                                          "attn_k.weight", "attn_v.weight", "attn_output.weight",
                                          "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};
    /* (ne0, ne1) of each: columns read per row, rows */
    const uint64_t shape[9][2] = {{dim, 1},     {dim, 1},  {dim, q_rows}, {dim, kv_rows}, {dim, kv_rows},
                                  {q_rows, dim}, {dim, ff}, {dim, ff},     {ff, dim}};
    const int L = d->n_layers;
    free(g->ptrs);
    free(g->norm_f32);
    g->ptrs = (const void **)calloc((size_t)9 * L, sizeof(void *));
    g->norm_f32 = NULL;
    if (!g->ptrs) return tos_set_status(TOS_ENOMEM);
    /* norms that are not F32 get a widened copy: count them first */
    size_t n_conv = 0;
    const gtensor_t *tn[9];
    for (int pass = 0; pass < 2; pass++) {
        size_t k = 0;
        if (pass == 1 && n_conv) {
            g->norm_f32 = (float *)malloc(n_conv * (size_t)d->dim * sizeof(float));
            if (!g->norm_f32) return tos_set_status(TOS_ENOMEM);
        }
        for (int l = 0; l < L; l++) {
            for (int j = 0; j < 9; j++) {
                char name[96];
                snprintf(name, sizeof(name), "blk.%d.%s", l, suffix[j]);
                int64_t i = tos_gguf_find_tensor(g, name);
                if (i < 0 || !tensor_is(&g->t[i], shape[j][0], shape[j][1])) return tos_set_status(TOS_EINVAL);
                tn[j] = &g->t[i];
                if (pass == 0) continue;
                if (j < 2 && tn[j]->type != 0) {
                    if (tn[j]->type != 1 || tn[j]->dims[0] != (uint64_t)d->dim) return tos_set_status(TOS_ENOTSUP);
                    float *dst = g->norm_f32 + k * (size_t)d->dim;
                    const uint8_t *src = (const uint8_t *)tn[j]->data;
                    for (int e = 0; e < d->dim; e++) dst[e] = fp16_to_f32((uint16_t)(src[2 * e] | (src[2 * e + 1] << 8)));
                    g->ptrs[(size_t)j * L + l] = dst;
                    k++;
                } else {
                    g->ptrs[(size_t)j * L + l] = tn[j]->data;
                }
            }
            if (pass == 0)
                for (int j = 0; j < 2; j++) n_conv += tn[j]->type != 0;
        }
    }
    /* every projection of one type (the device model's wtype) */
    int64_t iq = tos_gguf_find_tensor(g, "blk.0.attn_q.weight");
    d->wtype = (int)g->t[iq].type;
    for (int l = 0; l < L; l++)
        for (int j = 2; j < 9; j++) {
            char name[96];
            snprintf(name, sizeof(name), "blk.%d.%s", l, suffix[j]);
            if ((int)g->t[tos_gguf_find_tensor(g, name)].type != d->wtype) return tos_set_status(TOS_ENOTSUP);
        }
    /* output_norm: F32 or widened */
    const gtensor_t *on = &g->t[io];
    if (on->type == 0) {
        d->output_norm = (const float *)on->data;
    } else {
        return tos_set_status(TOS_ENOTSUP);
    }
    d->attn_norm = (const float *const *)(g->ptrs + 0 * (size_t)L);
    d->ffn_norm = (const float *const *)(g->ptrs + 1 * (size_t)L);
    d->wq = g->ptrs + 2 * (size_t)L;
    d->wk = g->ptrs + 3 * (size_t)L;
    d->wv = g->ptrs + 4 * (size_t)L;
    d->wo = g->ptrs + 5 * (size_t)L;
    d->wgate = g->ptrs + 6 * (size_t)L;
    d->wup = g->ptrs + 7 * (size_t)L;
    d->wdown = g->ptrs + 8 * (size_t)L;
    d->kv_type = TOS_TYPE_F16;
    return tos_set_status(TOS_OK);
}
