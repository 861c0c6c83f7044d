/*
 * laya_forward.c -- a plain C host for the B200 library: the sequence a
 * laya-zig maintainer's glue performs (INTEGRATION.md sections 2 and 3),
 * written against the C ABI alone.
 *
 *   loadModel (src/main.zig:2311-2404): map model.safetensors, read the
 *       8-byte header length and the JSON header (name -> dtype, shape,
 *       data_offsets), refuse a short or inconsistent file (BadSafetensors,
 *       main.zig:2321-2323), and hand every tensor to laya_gpu_create as a
 *       view of the mapping with its own dtype tag (the reference's matrices
 *       are F16, main.zig:1344-1362).
 *   forward (src/main.zig:2641-2817): laya_gpu_forward on one sequence, or
 *       laya_gpu_forward_dumpstats for --dumpstats (main.zig:113-130).
 *
 * usage: laya_forward MODEL QTYPE IDS MARKERS [--f16] [--dumpstats] [--device N]
 *   IDS and MARKERS are comma-separated lists ("-" for no markers).
 * Prints one JSON object {"logits": [...], "act": [a, e], "pooled": [768
 * values]} on stdout, or the [dump] text with --dumpstats. Exit status 0 on
 * success; 2 for a file that is not a safetensors image, 3 for a failed
 * laya_gpu_create, 4 for a failed forward, 1 for bad usage.
 */
#include <ctype.h>
#include <fcntl.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "laya_gpu.h"

/* ------------------------------------------------------------ header JSON */
/* A small reader for the safetensors header: an object whose values are
 * objects of strings, numbers and arrays ("__metadata__" holds strings). */
typedef struct {
    const char* p;
    const char* end;
    int bad;
} Rd;

static void skip_ws(Rd* r) {
    while (r->p < r->end && isspace((unsigned char)*r->p)) r->p++;
}

static int expect(Rd* r, char c) {
    skip_ws(r);
    if (r->p < r->end && *r->p == c) {
        r->p++;
        return 1;
    }
    r->bad = 1;
    return 0;
}

/* A JSON string into out (cap bytes, NUL-terminated); escapes other than
 * \" and \\ are kept as written (tensor names use neither). */
static int read_string(Rd* r, char* out, size_t cap) {
    size_t n = 0;
    if (!expect(r, '"')) return 0;
    while (r->p < r->end && *r->p != '"') {
        char ch = *r->p++;
        if (ch == '\\' && r->p < r->end) ch = *r->p++;
        if (n + 1 < cap) out[n++] = ch;
    }
    if (r->p >= r->end) {
        r->bad = 1;
        return 0;
    }
    r->p++;
    if (cap) out[n] = 0;
    return 1;
}

static int read_u64(Rd* r, uint64_t* v) {
    skip_ws(r);
    if (r->p >= r->end || !isdigit((unsigned char)*r->p)) {
        r->bad = 1;
        return 0;
    }
    uint64_t x = 0;
    while (r->p < r->end && isdigit((unsigned char)*r->p)) x = x * 10 + (uint64_t)(*r->p++ - '0');
    *v = x;
    return 1;
}

static void skip_value(Rd* r);

static void skip_composite(Rd* r, char open, char close) {
    r->p++; /* open */
    skip_ws(r);
    if (r->p < r->end && *r->p == close) {
        r->p++;
        return;
    }
    while (!r->bad) {
        if (open == '{') {
            char key[8];
            read_string(r, key, 0);
            expect(r, ':');
        }
        skip_value(r);
        skip_ws(r);
        if (r->p < r->end && *r->p == ',') {
            r->p++;
            continue;
        }
        expect(r, close);
        return;
    }
}

static void skip_value(Rd* r) {
    skip_ws(r);
    if (r->p >= r->end) {
        r->bad = 1;
        return;
    }
    const char c = *r->p;
    if (c == '"') {
        char tmp[8];
        read_string(r, tmp, 0);
    } else if (c == '{') {
        skip_composite(r, '{', '}');
    } else if (c == '[') {
        skip_composite(r, '[', ']');
    } else {
        while (r->p < r->end && (isalnum((unsigned char)*r->p) || *r->p == '-' || *r->p == '+' || *r->p == '.'))
            r->p++;
    }
}

typedef struct {
    char name[160];
    char dtype[16];
    uint64_t lo, hi;
} Entry;

/* Parses the header object into entries; returns their number, -1 if the
 * header is not the expected shape. */
static int parse_header(const char* hdr, size_t len, Entry** out) {
    Rd r = {hdr, hdr + len, 0};
    int n = 0, cap = 0;
    Entry* e = NULL;
    if (!expect(&r, '{')) return -1;
    skip_ws(&r);
    if (r.p < r.end && *r.p == '}') {
        *out = e;
        return 0;
    }
    while (!r.bad) {
        char key[160];
        if (!read_string(&r, key, sizeof key) || !expect(&r, ':')) break;
        if (strcmp(key, "__metadata__") == 0) {
            skip_value(&r);
        } else {
            if (n == cap) {
                cap = cap ? 2 * cap : 256;
                Entry* grown = (Entry*)realloc(e, (size_t)cap * sizeof(Entry));
                if (!grown) {
                    free(e);
                    return -1;
                }
                e = grown;
            }
            Entry* t = &e[n];
            memset(t, 0, sizeof *t);
            snprintf(t->name, sizeof t->name, "%s", key);
            int have_off = 0;
            if (!expect(&r, '{')) break;
            while (!r.bad) {
                char field[32];
                if (!read_string(&r, field, sizeof field) || !expect(&r, ':')) break;
                if (strcmp(field, "dtype") == 0) {
                    read_string(&r, t->dtype, sizeof t->dtype);
                } else if (strcmp(field, "data_offsets") == 0) {
                    if (expect(&r, '[') && read_u64(&r, &t->lo) && expect(&r, ',') && read_u64(&r, &t->hi) &&
                        expect(&r, ']'))
                        have_off = 1;
                } else {
                    skip_value(&r);
                }
                skip_ws(&r);
                if (r.p < r.end && *r.p == ',') {
                    r.p++;
                    continue;
                }
                expect(&r, '}');
                break;
            }
            if (!have_off || t->hi < t->lo) r.bad = 1;
            n++;
        }
        skip_ws(&r);
        if (r.p < r.end && *r.p == ',') {
            r.p++;
            continue;
        }
        expect(&r, '}');
        break;
    }
    if (r.bad) {
        free(e);
        return -1;
    }
    *out = e;
    return n;
}

/* ------------------------------------------------------------ arguments */
static uint32_t* parse_list(const char* s, uint32_t* n) {
    *n = 0;
    if (strcmp(s, "-") == 0) return NULL;
    uint32_t cap = 1;
    for (const char* q = s; *q; q++) cap += *q == ',';
    uint32_t* v = (uint32_t*)malloc(cap * sizeof(uint32_t));
    const char* q = s;
    while (v && *q) {
        char* end = NULL;
        const unsigned long x = strtoul(q, &end, 10);
        if (end == q) {
            free(v);
            return NULL;
        }
        v[(*n)++] = (uint32_t)x;
        q = *end == ',' ? end + 1 : end;
    }
    return v;
}

static int dtype_tag(const char* s) {
    if (strcmp(s, "F16") == 0) return LAYA_DT_F16;
    if (strcmp(s, "BF16") == 0) return LAYA_DT_BF16;
    if (strcmp(s, "F32") == 0) return LAYA_DT_F32;
    return -1; /* laya_gpu_create reports it if the model reads this tensor */
}

int main(int argc, char** argv) {
    if (argc < 5) {
        fprintf(stderr, "usage: %s MODEL QTYPE IDS MARKERS [--f16] [--dumpstats] [--device N]\n", argv[0]);
        return 1;
    }
    int precision = LAYA_PREC_BF16, dumpstats = 0, device = 0;
    for (int i = 5; i < argc; i++) {
        if (strcmp(argv[i], "--f16") == 0) precision = LAYA_PREC_F16;
        else if (strcmp(argv[i], "--dumpstats") == 0) dumpstats = 1;
        else if (strcmp(argv[i], "--device") == 0 && i + 1 < argc) device = atoi(argv[++i]);
        else {
            fprintf(stderr, "unknown option %s\n", argv[i]);
            return 1;
        }
    }
    const uint32_t qtype = (uint32_t)strtoul(argv[2], NULL, 10);
    uint32_t L = 0, K = 0;
    uint32_t* ids = parse_list(argv[3], &L);
    uint32_t* markers = parse_list(argv[4], &K);
    if (!ids || L == 0 || (strcmp(argv[4], "-") != 0 && !markers)) {
        fprintf(stderr, "bad IDS or MARKERS list\n");
        return 1;
    }

    /* loadModel: map the file, check the header bounds */
    const int fd = open(argv[1], O_RDONLY);
    struct stat st;
    if (fd < 0 || fstat(fd, &st) != 0) {
        fprintf(stderr, "cannot open %s\n", argv[1]);
        return 2;
    }
    const size_t size = (size_t)st.st_size;
    const uint8_t* data = size ? (const uint8_t*)mmap(NULL, size, PROT_READ, MAP_PRIVATE, fd, 0) : NULL;
    close(fd);
    if (size < 8 || data == (const uint8_t*)MAP_FAILED || !data) {
        fprintf(stderr, "error: BadSafetensors (file shorter than its 8-byte header length)\n");
        return 2;
    }
    uint64_t hdr_len = 0;
    for (int i = 7; i >= 0; i--) hdr_len = (hdr_len << 8) | data[i];
    if (hdr_len > size - 8) {
        fprintf(stderr, "error: BadSafetensors (header length %llu exceeds the file)\n", (unsigned long long)hdr_len);
        return 2;
    }
    const uint8_t* base = data + 8 + hdr_len;
    const size_t body = size - 8 - (size_t)hdr_len;
    Entry* ent = NULL;
    const int n = parse_header((const char*)data + 8, (size_t)hdr_len, &ent);
    if (n < 0) {
        fprintf(stderr, "error: BadSafetensors (header is not a safetensors JSON object)\n");
        return 2;
    }
    laya_tensor* t = (laya_tensor*)calloc(n ? (size_t)n : 1, sizeof(laya_tensor));
    for (int i = 0; i < n; i++) {
        if (ent[i].hi > body) {
            fprintf(stderr, "error: BadSafetensors (tensor %s runs past the end of the file)\n", ent[i].name);
            return 2;
        }
        const int tag = dtype_tag(ent[i].dtype);
        const uint64_t esz = tag == LAYA_DT_F32 ? 4 : 2;
        t[i].name = ent[i].name;
        t[i].dtype = tag;
        t[i].data = base + ent[i].lo;
        t[i].numel = (ent[i].hi - ent[i].lo) / esz;
    }

    laya_ctx* ctx = NULL;
    int rc = laya_gpu_create(device, t, n, precision, &ctx);
    if (rc != LAYA_OK) {
        fprintf(stderr, "laya_gpu_create: %s (status %d)\n", laya_gpu_last_error(NULL), rc);
        return 3;
    }
    munmap((void*)data, size); /* the library holds its own HBM copy */

    float* logits = (float*)calloc(K ? K : 1, sizeof(float));
    float act[2] = {0, 0};
    if (dumpstats) {
        uint64_t need = 0;
        rc = laya_gpu_forward_dumpstats(ctx, ids, L, qtype, markers, K, logits, act, NULL, 0, &need);
        if (rc == LAYA_ERR_ARG && need > 0) {
            char* text = (char*)malloc(need);
            rc = laya_gpu_forward_dumpstats(ctx, ids, L, qtype, markers, K, logits, act, text, need, NULL);
            if (rc == LAYA_OK) fputs(text, stdout);
            free(text);
        }
    } else {
        float* pooled = (float*)calloc(LAYA_HIDDEN, sizeof(float));
        rc = laya_gpu_forward(ctx, ids, L, qtype, markers, K, logits, act, pooled, NULL);
        if (rc == LAYA_OK) {
            printf("{\"logits\": [");
            for (uint32_t r = 0; r < K; r++) printf("%s%.9g", r ? ", " : "", logits[r]);
            printf("], \"act\": [%.9g, %.9g], \"pooled\": [", act[0], act[1]);
            for (int d = 0; d < LAYA_HIDDEN; d++) printf("%s%.9g", d ? ", " : "", pooled[d]);
            printf("]}\n");
        }
        free(pooled);
    }
    if (rc != LAYA_OK) {
        fprintf(stderr, "forward: %s (status %d)\n", laya_gpu_last_error(ctx), rc);
        laya_gpu_destroy(ctx);
        return 4;
    }
    laya_gpu_destroy(ctx);
    free(logits);
    free(t);
    free(ent);
    free(ids);
    free(markers);
    return 0;
}
