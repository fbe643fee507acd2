/*
 * oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of parakeet.cpp's f32 host decoder (the `use_graphs == false`
 * path of src/parakeet_tdt.cpp and the whole of src/parakeet_eou.cpp). It is the
 * checker for libparakeet_cuda and the timed CPU baseline; it is never linked
 * into or called by the product library. Only tests/, __graft_entry__.smoke()
 * and bench.py (cpu_baseline leg and --impl reference) use it.
 *
 * Parity pinning: the reference needs ggml (un-vendored, pin 58c38058 in
 * scripts/setup-ggml.sh:32) and cannot be compiled here, and its own decoder
 * fixtures need real GGUF models that are absent, so parity against outputs of
 * the reference itself is UNPINNED. What is pinned: (1) q8_0/f16
 * dequantization against gguf-py's `quants.dequantize` on the same bytes (the
 * quantizer library the reference's converter uses); (2) golden token/step
 * vectors under tests/golden/ produced by an independent float64 numpy
 * restatement of the same loop (tests/golden/make_golden.py).
 *
 * Built with the reference library's flags: -O3 -ffast-math -funroll-loops, no
 * -march (CMakeLists.txt:327-335).
 */
#ifndef PK_ORACLE_H
#define PK_ORACLE_H

#include "parakeet_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_model orc_model;

/* Host decoder state (TdtDecodeState src/parakeet_tdt.h:175-183 and
 * EouDecodeState src/parakeet_eou.h:53-66); arrays are caller-owned. */
typedef struct orc_state {
    float * h;            /* [L][H] */
    float * c;            /* [L][H] */
    float * pred;         /* [H]   */
    int32_t symbols_this_step;
    int32_t initialized;
    int32_t carry_frames;
    int32_t last_token;
    int32_t segment_start_token;
} orc_state;

/* Optional per-step trace. Any pointer may be NULL. Entries beyond max_steps
 * are not written (the decode itself continues). */
typedef struct orc_trace {
    int32_t   max_steps;
    float *   logits;       /* [max_steps][v_out] (TDT) or [max_steps][v_plus_1] (EOU) */
    float *   h;            /* [max_steps][L][H] state after the step */
    float *   c;            /* [max_steps][L][H] */
    int32_t * token;        /* [max_steps] argmax token */
    int32_t * dur_idx;      /* [max_steps] argmax duration index (TDT) */
    float *   margin_tok;   /* [max_steps] top1 - top2 over token logits */
    float *   margin_dur;   /* [max_steps] top1 - top2 over duration logits (TDT; +inf if 1 duration) */
    int32_t * frame;        /* [max_steps] frame index t evaluated at the step */
} orc_trace;

orc_model * orc_create(const pk_model_desc * desc, char * err, int32_t errlen);
void        orc_destroy(orc_model * m);

/* ggml to_float restated for F32 / F16 / Q8_0 rows: out gets ne0*ne1 floats. */
int32_t     orc_dequantize(const pk_tensor * t, float * out);

void        orc_dims(const orc_model * m, int32_t * dims8);  /* H, J, De, L, V+1, Vo, Nd, blank */

/* tdt_init_state (CPU branch, src/parakeet_tdt.cpp:813-863) and
 * eou_init_state (src/parakeet_eou.cpp:206-230). */
void        orc_init_state(const orc_model * m, orc_state * st);

/* tdt_decode_window (CPU branch, src/parakeet_tdt.cpp:865-981).
 * *n_tokens is in/out: the caller's running count on entry (tokens are written
 * from tokens[*n_tokens]), the new count on return. Returns the reference's rc
 * (0 ok, 1 d_model mismatch) or -1 if `cap` is exceeded. */
int32_t     orc_tdt_decode_window(const orc_model * m, const float * enc, int32_t n_frames,
                                  int32_t d_enc, int32_t max_symbols, orc_state * st,
                                  int32_t * tokens, int32_t cap, int32_t * n_tokens,
                                  int32_t * steps, orc_trace * trace);

/* eou_decode_window (src/parakeet_eou.cpp:232-336); same token conventions;
 * bounds[] receives EouSegmentBoundary::token_index values. */
int32_t     orc_eou_decode_window(const orc_model * m, const float * enc, int32_t n_frames,
                                  int32_t d_enc, int32_t max_symbols, orc_state * st,
                                  int32_t * tokens, int32_t cap, int32_t * n_tokens,
                                  int32_t * bounds, int32_t bounds_cap, int32_t * n_bounds,
                                  int32_t * steps, orc_trace * trace);

/* Greedy decode of B fresh utterances on n_threads host threads (one utterance
 * per thread at a time, weights shared read-only). Utterance b writes its
 * tokens at tokens[tok_region[b]...] (region capacity T_b * max_symbols) and
 * its count to n_tok[b]; EOU boundaries (if bounds != NULL) go to
 * bounds[bound_region[b]...] with counts in n_bounds[b]. ms[b] is the
 * utterance's wall time (first joint to last token, detokenize excluded).
 * Returns the wall time of the whole batch in ms, or a negative value on error. */
double      orc_decode_batch(const orc_model * m, const float * enc, const int64_t * frame_off,
                             const int32_t * n_frames, int32_t B, int32_t max_symbols,
                             int32_t n_threads, int32_t * tokens, const int64_t * tok_region,
                             int32_t * n_tok, int32_t * steps,
                             int32_t * bounds, const int64_t * bound_region, int32_t * n_bounds,
                             double * ms);

/* ctc_greedy_decode_window (src/parakeet_ctc.cpp:1831-1865): frames
 * [0, n_frames) of logits [n_frames][vocab_size]; *prev in/out. Tokens are
 * appended at tokens[*n_tokens] (and their frames at first_frame[*n_tokens] when
 * first_frame != NULL); returns -1 if `cap` would be exceeded, else 0. */
int32_t     orc_ctc_greedy_window(const float * logits, int32_t n_frames, int32_t vocab_size,
                                  int32_t blank_id, int32_t * prev, int32_t * tokens, int32_t cap,
                                  int32_t * n_tokens, int32_t * first_frame);

/* detokenize (src/sentencepiece_bpe.cpp:9-37) with a BpeVocab of n_pieces byte
 * strings (piece v = bytes[offsets[v] .. offsets[v + 1])). Writes at most `cap`
 * bytes of text; returns the text length (which may exceed cap). */
int64_t     orc_detokenize(const uint8_t * bytes, const int64_t * offsets, int32_t n_pieces,
                           int32_t blank_id, int32_t bos_id, int32_t eos_id, int32_t pad_id,
                           const int32_t * tokens, int64_t n_tokens, char * text, int64_t cap);

#ifdef __cplusplus
}
#endif

#endif
