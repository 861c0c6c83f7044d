/*
 * laya_tok.h -- C ABI of the host-side tokenizer and sequence builder that
 * feed the B200 forward pass (laya_gpu.h). Plain C++ on the host's cores:
 * tokenising many decisions runs on a pool of host threads and lands
 * directly in the packed batch layout laya_gpu_forward_device and
 * laya_gpu_forward_batch take.
 *
 * Reference interfaces replaced (paths within the laya-zig project):
 *
 *   laya_tok_load          loadTokenizer         src/main.zig:2045-2109
 *                          (walkValue / parseVocab / parseMerges / parseAdded
 *                          1717-1873, finishTokenizer 2000-2043)
 *   laya_tok_encode        encodeAll             src/main.zig:2197-2217
 *                          (encodeSegment 2162-2195, bpePiece 2111-2156)
 *   laya_tok_build         buildSequence         src/main.zig:2842-2911
 *                          (replaceMask 2820-2834, qtypeId 2914-2919)
 *   laya_tok_build_batch   the per-question loop of main (3747) and the
 *                          Snake move builder (3083), on host threads
 *
 * Results are identical to the reference's: same ids, same markers, same
 * truncation. Every call returns a laya_tok_status; after a failure,
 * laya_tok_last_error() (per calling thread) describes it. A loaded
 * tokenizer is immutable and may be used from any number of threads.
 */
#ifndef LAYA_TOK_H
#define LAYA_TOK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define LAYA_TOK_API __attribute__((visibility("default")))
#else
#define LAYA_TOK_API
#endif

/* Sequence builder constants (src/main.zig:50-57). */
#define LAYA_TOK_MAX_LEN 1024      /* default max_len of a built sequence */
#define LAYA_TOK_HEAD_MAX_LEN 256  /* default head_max_len */
#define LAYA_TOK_CLS_ID 2          /* <bos> */
#define LAYA_TOK_SEP_ID 1          /* <eos> */
#define LAYA_TOK_MASK_ID 4         /* <mask>: each option's marker token */
#define LAYA_TOK_OPT_MAX 48        /* tokens kept per option before its marker */

typedef enum {
    LAYA_TOK_OK = 0,
    LAYA_TOK_ERR_ARG = -1,       /* NULL pointer, head_max_len < 16, max_len == 0 */
    LAYA_TOK_ERR_IO = -2,        /* tokenizer.json cannot be read */
    LAYA_TOK_ERR_PARSE = -3,     /* malformed tokenizer.json (error.BadJson / TruncatedJson) */
    LAYA_TOK_ERR_QTYPE = -4,     /* question type not choice / score / noul (error.BadQuestionType) */
    LAYA_TOK_ERR_CAPACITY = -5,  /* an output array is too small; *n_out says how much is needed */
} laya_tok_status;

typedef struct laya_tok laya_tok;

/* Parse tokenizer.json at `path`: the "vocab", "merges" ([a, b] pairs,
 * ranked by position) and "added_tokens" keys wherever they appear. */
LAYA_TOK_API int laya_tok_load(const char* path, laya_tok** out);
LAYA_TOK_API void laya_tok_destroy(laya_tok* tok);
LAYA_TOK_API const char* laya_tok_last_error(void);

/* Table sizes: vocab entries, merges, added tokens. */
LAYA_TOK_API int laya_tok_sizes(const laya_tok* tok, uint32_t* vocab, uint32_t* merges, uint32_t* added);

/* encodeAll: `len` bytes of UTF-8 text -> token ids. *n_out receives the
 * count; if it exceeds `cap`, nothing past cap is written and the call
 * returns LAYA_TOK_ERR_CAPACITY. */
LAYA_TOK_API int laya_tok_encode(const laya_tok* tok, const char* text, size_t len, uint32_t* ids, size_t cap,
                                 size_t* n_out);

/* One decision: the state text, the question type name ("choice",
 * "score" or "noul"), the instruction and the option texts, all
 * NUL-terminated UTF-8. */
typedef struct {
    const char* state;
    const char* qtype_name;
    const char* ins;
    const char* const* opts;
    uint32_t n_opts;
} laya_decision;

/* buildSequence: [CLS] head [SEP] (<mask> option)* [SEP] state [SEP], cut
 * to max_len. ids needs max_len entries, markers n_opts; *L and *K receive
 * the lengths, *qtype the type id. */
LAYA_TOK_API int laya_tok_build(const laya_tok* tok, const laya_decision* d, uint32_t max_len, uint32_t head_max_len,
                                uint32_t* ids, uint32_t* L, uint32_t* markers, uint32_t* K, uint32_t* qtype);

/* Many decisions at once on `threads` host threads (0 = one per core, at
 * most 8, as the reference's pool defaults: src/main.zig:3588-3597), packed
 * back to back as laya_batch expects: ids[n_tokens], cu_seqlens[n + 1],
 * markers[n_markers] (positions within their sequence), cu_markers[n + 1],
 * qtypes[n]. ids_cap / markers_cap bound the two variable-size arrays; on
 * LAYA_TOK_ERR_CAPACITY *n_tokens / *n_markers say how much is needed.
 * Results do not depend on the thread count. */
LAYA_TOK_API int laya_tok_build_batch(const laya_tok* tok, const laya_decision* d, uint32_t n, uint32_t max_len,
                                      uint32_t head_max_len, int threads, uint32_t* ids, size_t ids_cap,
                                      int32_t* cu_seqlens, uint32_t* markers, size_t markers_cap,
                                      int32_t* cu_markers, uint32_t* qtypes, size_t* n_tokens, size_t* n_markers);

#ifdef __cplusplus
}
#endif

#endif /* LAYA_TOK_H */
