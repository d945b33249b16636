/* k3_ckpt.c -- safetensors checkpoint index for loading released weights into HBM.
 *
 * The reference reads its checkpoint through src/io/k3_st.c (index), src/model/k3_bind.c
 * (names, element-count validation, 167-241) and src/io/k3_load.c (expert checks and the
 * contiguous six-tensor run, 46-103). This is the device loader's counterpart: it indexes
 * every *.safetensors file of a directory (an 8-byte little-endian header length, a JSON
 * header of {name: {dtype, shape, data_offsets}}, offsets relative to the end of the
 * header), answers lookups by name through an open-addressed hash table, and reads byte
 * ranges with pread. k3d_model_load_checkpoint (k3_stack.c) binds the tensors to the
 * decode stack and uploads them.
 *
 * Every entry is validated when the header is read: a known dtype, at most four
 * dimensions, end >= start, the span equal to the element count times the element size,
 * and the span inside the file. A header that fails any of these refuses the whole
 * directory: a silently misread tensor is a model that runs and is wrong.
 */
#define _POSIX_C_SOURCE 200809L
#define _FILE_OFFSET_BITS 64

#include <dirent.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include "k3_cuda.h"

typedef struct {
    char *name;
    K3dCkptTensor t;
} Entry;

struct K3dCkpt {
    int *fd;
    int nshard;
    Entry *e;
    int ne, cap;
    int32_t *bucket;                /* open addressing, -1 empty */
    int nbucket;
};

static char g_err[512];

static void set_err(const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

const char *k3d_ckpt_error(void) { return g_err; }

/* for the binder in k3_stack.c */
void k3h_ckpt_fail(const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

int k3d_ckpt_elem_size(int dtype)
{
    switch (dtype) {
    case K3D_DT_U8: return 1;
    case K3D_DT_BF16:
    case K3D_DT_F16: return 2;
    case K3D_DT_F32: return 4;
    default: return 0;
    }
}

static int dtype_code(const char *s, size_t n)
{
    if (n == 2 && !memcmp(s, "U8", 2)) return K3D_DT_U8;
    if (n == 4 && !memcmp(s, "BF16", 4)) return K3D_DT_BF16;
    if (n == 3 && !memcmp(s, "F16", 3)) return K3D_DT_F16;
    if (n == 3 && !memcmp(s, "F32", 3)) return K3D_DT_F32;
    return 0;
}

static uint64_t name_hash(const char *s)
{
    uint64_t h = 0xcbf29ce484222325ull;          /* FNV-1a over every byte of the name */
    for (; *s; s++) {
        h ^= (unsigned char)*s;
        h *= 0x100000001b3ull;
    }
    return h;
}

/* ------------------------------------------------------------- JSON scanner
 * The header is one flat object whose values are objects with the keys dtype, shape and
 * data_offsets (plus an optional "__metadata__" object of strings, skipped). */
typedef struct {
    const char *p, *end;
} Scan;

static void ws(Scan *s)
{
    while (s->p < s->end && (*s->p == ' ' || *s->p == '\n' || *s->p == '\r' || *s->p == '\t')) s->p++;
}

static int expect(Scan *s, char c)
{
    ws(s);
    if (s->p >= s->end || *s->p != c) return -1;
    s->p++;
    return 0;
}

/* A JSON string into a fresh allocation (escapes \" \\ \/ kept as the character; any
 * other escape is refused: tensor names never need them). */
static char *str(Scan *s, size_t *len)
{
    ws(s);
    if (s->p >= s->end || *s->p != '"') return NULL;
    s->p++;
    const char *b = s->p;
    size_t n = 0;
    for (const char *q = b; q < s->end && *q != '"'; q++, n++)
        if (*q == '\\') q++;
    char *out = (char *)malloc(n + 1);
    if (!out) return NULL;
    size_t k = 0;
    while (s->p < s->end && *s->p != '"') {
        char c = *s->p++;
        if (c == '\\') {
            if (s->p >= s->end) { free(out); return NULL; }
            c = *s->p++;
            if (c != '"' && c != '\\' && c != '/') { free(out); return NULL; }
        }
        out[k++] = c;
    }
    if (s->p >= s->end) { free(out); return NULL; }
    s->p++;
    out[k] = 0;
    if (len) *len = k;
    return out;
}

static int integer(Scan *s, int64_t *v)
{
    ws(s);
    if (s->p >= s->end || *s->p < '0' || *s->p > '9') return -1;
    int64_t x = 0;
    while (s->p < s->end && *s->p >= '0' && *s->p <= '9') {
        if (x > (INT64_MAX - 9) / 10) return -1;
        x = x * 10 + (*s->p++ - '0');
    }
    *v = x;
    return 0;
}

static int int_list(Scan *s, int64_t *v, int maxn, int *n)
{
    if (expect(s, '[')) return -1;
    *n = 0;
    ws(s);
    if (s->p < s->end && *s->p == ']') { s->p++; return 0; }
    for (;;) {
        int64_t x;
        if (integer(s, &x)) return -1;
        if (*n >= maxn) return -1;
        v[(*n)++] = x;
        ws(s);
        if (s->p < s->end && *s->p == ',') { s->p++; continue; }
        return expect(s, ']');
    }
}

/* skips any value whose objects and arrays hold only strings, numbers and nesting */
static int skip_value(Scan *s, int depth)
{
    if (depth > 16) return -1;
    ws(s);
    if (s->p >= s->end) return -1;
    if (*s->p == '"') {
        char *t = str(s, NULL);
        if (!t) return -1;
        free(t);
        return 0;
    }
    if (*s->p == '{' || *s->p == '[') {
        const char close = *s->p == '{' ? '}' : ']';
        const int obj = *s->p == '{';
        s->p++;
        ws(s);
        if (s->p < s->end && *s->p == close) { s->p++; return 0; }
        for (;;) {
            if (obj) {
                char *k = str(s, NULL);
                if (!k) return -1;
                free(k);
                if (expect(s, ':')) return -1;
            }
            if (skip_value(s, depth + 1)) return -1;
            ws(s);
            if (s->p < s->end && *s->p == ',') { s->p++; continue; }
            return expect(s, close);
        }
    }
    while (s->p < s->end && *s->p != ',' && *s->p != '}' && *s->p != ']') s->p++;   /* number, literal */
    return 0;
}

static int add_entry(K3dCkpt *c, char *name, const K3dCkptTensor *t)
{
    if (c->ne == c->cap) {
        const int nc = c->cap ? 2 * c->cap : 1024;
        Entry *e = (Entry *)realloc(c->e, (size_t)nc * sizeof(Entry));
        if (!e) return -1;
        c->e = e;
        c->cap = nc;
    }
    c->e[c->ne].name = name;
    c->e[c->ne].t = *t;
    c->ne++;
    return 0;
}

static int index_shard(K3dCkpt *c, int shard, const char *path)
{
    const int fd = c->fd[shard];
    struct stat st;
    unsigned char lenb[8];
    if (fstat(fd, &st) || pread(fd, lenb, 8, 0) != 8) { set_err("%s: unreadable", path); return -1; }
    uint64_t hl = 0;
    for (int i = 7; i >= 0; i--) hl = (hl << 8) | lenb[i];
    const int64_t fsize = (int64_t)st.st_size;
    if (hl == 0 || hl > (uint64_t)fsize - 8 || hl > ((uint64_t)1 << 31)) {
        set_err("%s: header length %llu does not fit the file", path, (unsigned long long)hl);
        return -1;
    }
    char *h = (char *)malloc(hl);
    if (!h || pread(fd, h, hl, 8) != (ssize_t)hl) { free(h); set_err("%s: short header", path); return -1; }
    Scan s = {h, h + hl};
    const int64_t base = 8 + (int64_t)hl;
    int rc = expect(&s, '{');
    ws(&s);
    if (!rc && s.p < s.end && *s.p == '}') s.p++;
    else while (!rc) {
        char *name = str(&s, NULL);
        if (!name || expect(&s, ':')) { free(name); rc = -1; break; }
        if (!strcmp(name, "__metadata__")) {
            free(name);
            if (skip_value(&s, 0)) { rc = -1; break; }
        } else {
            K3dCkptTensor t;
            memset(&t, 0, sizeof t);
            t.shard = shard;
            int64_t offs[2];
            int noff = -1, have_dt = 0, have_shape = 0;
            if (expect(&s, '{')) { free(name); rc = -1; break; }
            for (;;) {
                size_t kl;
                char *k = str(&s, &kl);
                if (!k || expect(&s, ':')) { free(k); rc = -1; break; }
                if (!strcmp(k, "dtype")) {
                    size_t dl;
                    char *d = str(&s, &dl);
                    t.dtype = d ? dtype_code(d, dl) : 0;
                    free(d);
                    have_dt = 1;
                } else if (!strcmp(k, "shape")) {
                    int nd;
                    if (int_list(&s, t.shape, 4, &nd)) { free(k); rc = -1; break; }
                    t.ndim = nd;
                    have_shape = 1;
                } else if (!strcmp(k, "data_offsets")) {
                    if (int_list(&s, offs, 2, &noff) || noff != 2) { free(k); rc = -1; break; }
                } else if (skip_value(&s, 0)) {
                    free(k);
                    rc = -1;
                    break;
                }
                free(k);
                ws(&s);
                if (s.p < s.end && *s.p == ',') { s.p++; continue; }
                if (expect(&s, '}')) rc = -1;
                break;
            }
            if (rc) { free(name); set_err("%s: malformed header entry", path); break; }
            if (!have_dt || !have_shape || noff != 2 || !t.dtype) {
                set_err("%s: %s: missing or unknown dtype, shape or data_offsets", path, name);
                free(name);
                rc = -1;
                break;
            }
            int64_t numel = 1;
            for (int i = 0; i < t.ndim; i++) {
                if (t.shape[i] && numel > INT64_MAX / t.shape[i]) { numel = -1; break; }
                numel *= t.shape[i];
            }
            t.off = base + offs[0];
            t.nbytes = offs[1] - offs[0];
            if (numel < 0 || offs[1] < offs[0] || t.nbytes != numel * k3d_ckpt_elem_size(t.dtype) ||
                t.off + t.nbytes > fsize) {
                set_err("%s: %s: data_offsets [%lld, %lld) do not hold its shape or leave the file", path,
                        name, (long long)offs[0], (long long)offs[1]);
                free(name);
                rc = -1;
                break;
            }
            if (add_entry(c, name, &t)) { free(name); rc = -1; break; }
        }
        ws(&s);
        if (s.p < s.end && *s.p == ',') { s.p++; continue; }
        if (expect(&s, '}')) { set_err("%s: malformed header", path); rc = -1; }
        break;
    }
    if (rc && !g_err[0]) set_err("%s: malformed header", path);
    free(h);
    return rc;
}

static int cmp_names(const void *a, const void *b)
{
    return strcmp(*(char *const *)a, *(char *const *)b);
}

void k3d_ckpt_close(K3dCkpt *c)
{
    if (!c) return;
    for (int i = 0; i < c->nshard; i++)
        if (c->fd[i] >= 0) close(c->fd[i]);
    for (int i = 0; i < c->ne; i++) free(c->e[i].name);
    free(c->fd);
    free(c->e);
    free(c->bucket);
    free(c);
}

K3dCkpt *k3d_ckpt_open(const char *dir)
{
    g_err[0] = 0;
    if (!dir) { set_err("null directory"); return NULL; }
    DIR *d = opendir(dir);
    if (!d) { set_err("%s: cannot open directory", dir); return NULL; }
    char **files = NULL;
    int nf = 0, capf = 0;
    struct dirent *de;
    while ((de = readdir(d))) {
        const size_t n = strlen(de->d_name);
        if (n > 12 && !strcmp(de->d_name + n - 12, ".safetensors")) {
            if (nf == capf) {
                capf = capf ? 2 * capf : 16;
                char **f2 = (char **)realloc(files, (size_t)capf * sizeof(char *));
                if (!f2) break;
                files = f2;
            }
            files[nf] = (char *)malloc(strlen(dir) + n + 2);
            if (!files[nf]) break;
            sprintf(files[nf], "%s/%s", dir, de->d_name);
            nf++;
        }
    }
    closedir(d);
    K3dCkpt *c = (K3dCkpt *)calloc(1, sizeof *c);
    if (!c || !nf) {
        if (!nf) set_err("%s: no .safetensors files", dir);
        for (int i = 0; i < nf; i++) free(files[i]);
        free(files);
        free(c);
        return NULL;
    }
    qsort(files, (size_t)nf, sizeof(char *), cmp_names);      /* shard order = file name order */
    c->fd = (int *)malloc((size_t)nf * sizeof(int));
    int rc = c->fd ? 0 : -1;
    for (int i = 0; i < nf && !rc; i++) {
        c->fd[i] = open(files[i], O_RDONLY);
        c->nshard = i + 1;
        if (c->fd[i] < 0) { set_err("%s: cannot open", files[i]); rc = -1; break; }
        rc = index_shard(c, i, files[i]);
    }
    for (int i = 0; i < nf; i++) free(files[i]);
    free(files);
    if (!rc) {
        c->nbucket = 16;
        while (c->nbucket < 2 * c->ne) c->nbucket *= 2;
        c->bucket = (int32_t *)malloc((size_t)c->nbucket * sizeof(int32_t));
        if (!c->bucket) rc = -1;
        for (int i = 0; !rc && i < c->nbucket; i++) c->bucket[i] = -1;
        for (int i = 0; !rc && i < c->ne; i++) {
            size_t b = (size_t)(name_hash(c->e[i].name) & (uint64_t)(c->nbucket - 1));
            while (c->bucket[b] >= 0) {
                if (!strcmp(c->e[c->bucket[b]].name, c->e[i].name)) {
                    set_err("tensor %s appears twice", c->e[i].name);
                    rc = -1;
                    break;
                }
                b = (b + 1) & (size_t)(c->nbucket - 1);
            }
            if (!rc) c->bucket[b] = i;
        }
    }
    if (rc) { k3d_ckpt_close(c); return NULL; }
    return c;
}

int k3d_ckpt_count(const K3dCkpt *c) { return c ? c->ne : 0; }

int k3d_ckpt_find(const K3dCkpt *c, const char *name, K3dCkptTensor *out)
{
    if (!c || !name || !c->nbucket) return K3D_EINVAL;
    size_t b = (size_t)(name_hash(name) & (uint64_t)(c->nbucket - 1));
    while (c->bucket[b] >= 0) {
        const Entry *e = &c->e[c->bucket[b]];
        if (!strcmp(e->name, name)) {
            if (out) *out = e->t;
            return K3D_OK;
        }
        b = (b + 1) & (size_t)(c->nbucket - 1);
    }
    return K3D_EINVAL;
}

int64_t k3d_ckpt_read(const K3dCkpt *c, int shard, int64_t off, int64_t nbytes, void *buf)
{
    if (!c || shard < 0 || shard >= c->nshard || off < 0 || nbytes < 0 || (nbytes && !buf)) return -1;
    int64_t done = 0;
    while (done < nbytes) {
        const ssize_t r = pread(c->fd[shard], (char *)buf + done, (size_t)(nbytes - done), (off_t)(off + done));
        if (r <= 0) return done;
        done += r;
    }
    return done;
}
