/* gguf.c -- the routed-expert tensors of the engine's GGUF model file, for the HBM expert pool.
 *
 * The reference engine opens its model with gguf_open (src/gguf.c:80-160: GGUF v2/v3 container, typed key/values,
 * tensor infos, tensor data at the header's end rounded up to "general.alignment", each tensor's size taken as the
 * distance to the next tensor's offset) and setup_experts (src/engine.c:336-351) then reads "inz.expert_type",
 * "inz.expert_blob_bytes" and, per layer, "blk.%d.experts" (the MTP layer's "mtp.experts" comes after the last layer).
 * This reader keeps only that: one pass over the header that skips every other value and records the expert tensors
 * by layer. The file stays mapped read-only until inzg_gguf_close, so a layer's blobs go to the pool straight from the
 * page cache (inzg_pool_add_layer_gguf) without a second host copy. Host code only.
 */
#define _GNU_SOURCE
#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "../../../include/inzg.h"

enum { KV_U8 = 0, KV_I8 = 1, KV_U16 = 2, KV_I16 = 3, KV_U32 = 4, KV_I32 = 5, KV_F32 = 6, KV_BOOL = 7, KV_STR = 8,
       KV_ARR = 9, KV_U64 = 10, KV_I64 = 11, KV_F64 = 12 };

#define GGUF_MAGIC 0x46554747u /* "GGUF" */
#define MAX_LAYERS 4096
#define NO_TENSOR UINT64_MAX

struct inzg_gguf {
    int fd;
    uint8_t *map;
    size_t size;
    inzg_gguf_info info;
    uint64_t layer_off[MAX_LAYERS + 1], layer_len[MAX_LAYERS + 1]; /* [MAX_LAYERS]: mtp.experts */
};

typedef struct {
    const uint8_t *p, *end;
    int ok;
} cursor;

static uint64_t take(cursor *c, size_t n) { /* little-endian unsigned of n <= 8 bytes */
    uint64_t v = 0;
    if (!c->ok || (size_t)(c->end - c->p) < n) {
        c->ok = 0;
        return 0;
    }
    memcpy(&v, c->p, n);
    c->p += n;
    return v;
}

/* a length-prefixed string: its bytes stay in the mapping */
static const char *take_str(cursor *c, uint64_t *len) {
    *len = take(c, 8);
    if (!c->ok || (uint64_t)(c->end - c->p) < *len) {
        c->ok = 0;
        return NULL;
    }
    const char *s = (const char *)c->p;
    c->p += *len;
    return s;
}

static size_t scalar_bytes(uint32_t t) {
    switch (t) {
    case KV_U8: case KV_I8: case KV_BOOL: return 1;
    case KV_U16: case KV_I16: return 2;
    case KV_U32: case KV_I32: case KV_F32: return 4;
    case KV_U64: case KV_I64: case KV_F64: return 8;
    default: return 0;
    }
}

static int skip(cursor *c, uint32_t t, int depth) {
    if (depth > 8) return c->ok = 0;
    if (t == KV_STR) {
        uint64_t n;
        take_str(c, &n);
        return c->ok;
    }
    if (t == KV_ARR) {
        const uint32_t et = (uint32_t)take(c, 4);
        const uint64_t n = take(c, 8);
        if (!c->ok) return 0;
        if (et == KV_STR || et == KV_ARR) {
            for (uint64_t i = 0; i < n && c->ok; i++) skip(c, et, depth + 1);
            return c->ok;
        }
        const size_t es = scalar_bytes(et);
        if (!es || (uint64_t)(c->end - c->p) / es < n) return c->ok = 0;
        c->p += es * n;
        return 1;
    }
    const size_t es = scalar_bytes(t);
    if (!es) return c->ok = 0;
    take(c, es);
    return c->ok;
}

/* an integer-valued key as gguf_get_int reads it (src/gguf.c:189-199): signed, unsigned, bool or float scalars */
static int scalar_int(cursor *c, uint32_t t, int64_t *out) {
    const size_t es = scalar_bytes(t);
    if (!es) return 0;
    const uint64_t u = take(c, es);
    if (!c->ok) return 0;
    switch (t) {
    case KV_I8: *out = (int8_t)u; break;
    case KV_I16: *out = (int16_t)u; break;
    case KV_I32: *out = (int32_t)u; break;
    case KV_I64: *out = (int64_t)u; break;
    case KV_F32: { float f; uint32_t b = (uint32_t)u; memcpy(&f, &b, 4); *out = (int64_t)f; break; }
    case KV_F64: { double f; memcpy(&f, &u, 8); *out = (int64_t)f; break; }
    case KV_BOOL: *out = u != 0; break;
    default: *out = (int64_t)u; break;
    }
    return 1;
}

static int key_is(const char *k, uint64_t n, const char *want) { return n == strlen(want) && !memcmp(k, want, n); }

/* "blk.<layer>.experts" (decimal, as snprintf("%d") writes it) -> layer, "mtp.experts" -> MAX_LAYERS, else -1 */
static int expert_layer(const char *s, uint64_t n) {
    if (key_is(s, n, "mtp.experts")) return MAX_LAYERS;
    static const char pre[] = "blk.", suf[] = ".experts";
    const uint64_t np = sizeof(pre) - 1, ns = sizeof(suf) - 1;
    if (n <= np + ns || memcmp(s, pre, np) || memcmp(s + n - ns, suf, ns)) return -1;
    const char *d = s + np;
    const uint64_t nd = n - np - ns;
    if (nd > 4 || (nd > 1 && d[0] == '0')) return -1;
    int v = 0;
    for (uint64_t i = 0; i < nd; i++) {
        if (d[i] < '0' || d[i] > '9') return -1;
        v = v * 10 + (d[i] - '0');
    }
    return v < MAX_LAYERS ? v : -1;
}

static int cmp_u64(const void *a, const void *b) {
    const uint64_t x = *(const uint64_t *)a, y = *(const uint64_t *)b;
    return x < y ? -1 : x > y;
}

static void set_err(char *err, size_t len, const char *fmt, ...) {
    if (!err || !len) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, len, fmt, ap);
    va_end(ap);
}

INZG_EXPORT void inzg_gguf_close(inzg_gguf *g) {
    if (!g) return;
    if (g->map) munmap(g->map, g->size);
    if (g->fd >= 0) close(g->fd);
    free(g);
}

INZG_EXPORT inzg_gguf *inzg_gguf_open(const char *path, inzg_gguf_info *info, char *err, size_t err_len) {
    if (!path) {
        set_err(err, err_len, "gguf: no path");
        return NULL;
    }
    inzg_gguf *g = calloc(1, sizeof(*g));
    if (!g) {
        set_err(err, err_len, "gguf: out of host memory");
        return NULL;
    }
    g->fd = open(path, O_RDONLY | O_CLOEXEC);
    struct stat st;
    if (g->fd < 0 || fstat(g->fd, &st) != 0) {
        set_err(err, err_len, "gguf: open %s: %s", path, strerror(errno));
        inzg_gguf_close(g);
        return NULL;
    }
    g->size = (size_t)st.st_size;
    if (g->size < 24) {
        set_err(err, err_len, "gguf: %s is not a GGUF file", path);
        inzg_gguf_close(g);
        return NULL;
    }
    void *m = mmap(NULL, g->size, PROT_READ, MAP_SHARED, g->fd, 0);
    if (m == MAP_FAILED) {
        set_err(err, err_len, "gguf: mmap %s: %s", path, strerror(errno));
        inzg_gguf_close(g);
        return NULL;
    }
    g->map = m;
    for (int l = 0; l <= MAX_LAYERS; l++) g->layer_off[l] = NO_TENSOR;

    cursor c = {g->map, g->map + g->size, 1};
    const char *why = NULL;
    uint64_t *offs = NULL;
    int64_t etype = INZG_T_Q8G, blob = 0, align = 32; /* the engine's defaults (src/engine.c:338-339, gguf.c:98) */
    if ((uint32_t)take(&c, 4) != GGUF_MAGIC) { why = "not a GGUF file"; goto bad; }
    const uint32_t version = (uint32_t)take(&c, 4);
    if (version < 2 || version > 3) { why = "GGUF version other than 2 or 3"; goto bad; }
    const uint64_t n_tensors = take(&c, 8), n_kv = take(&c, 8);
    if (!c.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) { why = "bad header counts"; goto bad; }
    for (uint64_t i = 0; i < n_kv; i++) {
        uint64_t kn;
        const char *k = take_str(&c, &kn);
        const uint32_t t = (uint32_t)take(&c, 4);
        if (!c.ok) { why = "truncated key/value section"; goto bad; }
        int64_t *dst = key_is(k, kn, "inz.expert_type") ? &etype
                       : key_is(k, kn, "inz.expert_blob_bytes") ? &blob
                       : key_is(k, kn, "general.alignment") ? &align : NULL;
        if (dst && scalar_bytes(t)) {
            if (!scalar_int(&c, t, dst)) { why = "truncated key/value section"; goto bad; }
        } else if (!skip(&c, t, 0)) {
            why = "bad or truncated key/value";
            goto bad;
        }
    }
    if (align <= 0) align = 32;  /* alignment 0 means the default (src/gguf.c:132) */
    offs = malloc(sizeof(uint64_t) * (n_tensors ? n_tensors : 1));
    if (!offs) { why = "out of host memory"; goto bad; }
    for (uint64_t i = 0; i < n_tensors; i++) {
        uint64_t nn;
        const char *name = take_str(&c, &nn);
        const uint32_t nd = (uint32_t)take(&c, 4);
        if (!c.ok || nd > 4) { why = "bad or truncated tensor info"; goto bad; }
        for (uint32_t d = 0; d < nd; d++) take(&c, 8);
        take(&c, 4);  /* tensor type */
        offs[i] = take(&c, 8);
        if (!c.ok) { why = "truncated tensor info"; goto bad; }
        const int l = expert_layer(name, nn);
        if (l >= 0) g->layer_off[l] = offs[i];
    }
    const uint64_t hdr = (uint64_t)(c.p - g->map);
    const uint64_t data = (hdr + (uint64_t)align - 1) / (uint64_t)align * (uint64_t)align;
    if (data > g->size) { why = "tensor data section beyond the end of the file"; goto bad; }
    qsort(offs, n_tensors, sizeof(uint64_t), cmp_u64);
    for (int l = 0; l <= MAX_LAYERS; l++) {
        const uint64_t o = g->layer_off[l];
        if (o == NO_TENSOR) continue;
        if (o > g->size - data) { why = "expert tensor beyond the end of the file"; goto bad; }
        /* size: up to the next tensor's offset, the last one up to the end of the file (src/gguf.c:148-156) */
        uint64_t end = g->size - data;
        size_t lo = 0, hi = n_tensors;
        while (lo < hi) {  /* first offset > o */
            const size_t mid = (lo + hi) / 2;
            if (offs[mid] <= o) lo = mid + 1;
            else hi = mid;
        }
        if (lo < n_tensors && offs[lo] < end) end = offs[lo];
        g->layer_len[l] = end - o;
        g->layer_off[l] = data + o;  /* absolute */
    }
    free(offs);
    g->info.expert_type = (int)etype;
    g->info.blob_bytes = blob > 0 ? (uint64_t)blob : 0;
    g->info.alignment = (uint64_t)align;
    g->info.data_offset = data;
    while (g->info.n_layers < MAX_LAYERS && g->layer_off[g->info.n_layers] != NO_TENSOR) g->info.n_layers++;
    g->info.has_mtp = g->layer_off[MAX_LAYERS] != NO_TENSOR;
    if (info) *info = g->info;
    return g;
bad:
    set_err(err, err_len, "gguf: %s: %s", path, why);
    free(offs);
    inzg_gguf_close(g);
    return NULL;
}

INZG_EXPORT inzg_status inzg_gguf_get_info(const inzg_gguf *g, inzg_gguf_info *info) {
    if (!g || !info) return INZG_BAD_ARG;
    *info = g->info;
    return INZG_OK;
}

INZG_EXPORT inzg_status inzg_gguf_experts(const inzg_gguf *g, int layer, const void **data, uint64_t *nbytes,
                                          uint64_t *file_offset) {
    if (!g || layer < 0) return INZG_BAD_ARG;
    int slot = -1;
    if (layer < g->info.n_layers) slot = layer;
    else if (layer == g->info.n_layers && g->info.has_mtp) slot = MAX_LAYERS;
    if (slot < 0) return INZG_BAD_ARG;
    if (data) *data = g->map + g->layer_off[slot];
    if (nbytes) *nbytes = g->layer_len[slot];
    if (file_offset) *file_offset = g->layer_off[slot];
    return INZG_OK;
}
