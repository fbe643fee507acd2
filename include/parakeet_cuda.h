/*
 * parakeet_cuda.h -- C ABI of libparakeet_cuda, the B200 (sm_100a) greedy
 * transducer decoder for parakeet.cpp's TDT and RNN-T/EOU token loops.
 *
 * The library replaces the decoder dispatch of parakeet.cpp (the reference):
 *   - tdt_prepare_runtime   src/parakeet_tdt.cpp:585-718  -> pk_create
 *   - tdt_init_state        src/parakeet_tdt.cpp:813-863  -> pk_stream_reset
 *   - tdt_decode_window     src/parakeet_tdt.cpp:865-981  -> pk_stream_window
 *   - tdt_greedy_decode     src/parakeet_tdt.cpp:983-1005 -> pk_decode_batch (B >= 1)
 *   - eou_prepare_runtime   src/parakeet_eou.cpp:172-204  -> pk_create (PK_MODEL_EOU)
 *   - eou_init_state        src/parakeet_eou.cpp:206-230  -> pk_stream_reset
 *   - eou_decode_window     src/parakeet_eou.cpp:232-336  -> pk_stream_window
 *   - eou_greedy_decode     src/parakeet_eou.cpp:338-387  -> pk_decode_batch
 *
 * Conventions (mirroring the reference's int return codes, parakeet_tdt.h:185-205):
 *   - every entry point returns a pk_status; 0 is success, nothing aborts;
 *   - pk_last_error() returns a thread-local message for the last failure;
 *   - weights are passed as raw GGUF tensor blocks (ggml type F32 / F16 / Q8_0,
 *     row-major [ne1][ne0] with ne0 = input features contiguous, the layout the
 *     converter writes in scripts/convert-nemo-to-gguf.py:405-413); the library
 *     copies and repacks them once; the caller keeps ownership of its buffers;
 *   - encoder output is f32 [T][d_enc] row-major, on the host or on the device;
 *   - one context per device; calls on one context are not concurrent
 *     (same rule as parakeet::Engine, include/parakeet/engine.h:35-55).
 *
 * No C++ or torch types cross this boundary.
 */
#ifndef PARAKEET_CUDA_H
#define PARAKEET_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PK_ABI_VERSION 1

#if defined(__GNUC__) || defined(__clang__)
#define PK_API __attribute__((visibility("default")))
#else
#define PK_API
#endif

typedef enum pk_status {
    PK_OK             = 0,
    PK_ERR_DMODEL     = 1,  /* encoder d_model mismatch (tdt_decode_window rc 1, parakeet_tdt.cpp:874-878) */
    PK_ERR_INVALID    = 2,  /* null pointer, negative size, bad option */
    PK_ERR_MODEL      = 3,  /* missing tensor, wrong shape, unsupported ggml type */
    PK_ERR_CUDA       = 4,  /* CUDA runtime error (message in pk_last_error) */
    PK_ERR_OOM        = 5,  /* device allocation failed */
    PK_ERR_TIMEOUT    = 6,  /* a bounded device-side wait (grid barrier) ran out */
    PK_ERR_CAPACITY   = 7,  /* caller's output buffer too small; *_needed fields hold the size */
    PK_ERR_NO_DEVICE  = 8,  /* no CUDA device / not sm_100 */
    PK_ERR_DEVICE     = 9   /* a device-side index check failed (bad token / frame index) */
} pk_status;

/* ggml tensor type ids accepted in pk_tensor.type (values of enum ggml_type). */
enum { PK_GGML_F32 = 0, PK_GGML_F16 = 1, PK_GGML_Q8_0 = 8 };

/* Decoder families (ParakeetModelType, src/parakeet_ctc.h:225-230). */
enum { PK_MODEL_TDT = 1, PK_MODEL_EOU = 2 };

/* One GGUF tensor: raw blocks exactly as stored in the file / ggml tensor.
 * 2-D weights: ne0 = in_features (contiguous), ne1 = out_features.
 * 1-D biases: ne0 = length, ne1 = 1. */
typedef struct pk_tensor {
    const void * data;
    int32_t      type;     /* PK_GGML_* */
    int32_t      reserved;
    int64_t      ne0;
    int64_t      ne1;
    uint64_t     nbytes;
} pk_tensor;

/* One prediction-net LSTM layer (TdtLstmLayer, src/parakeet_ctc.h:180-185);
 * GGUF names {tdt,eou}.predict.lstm.<l>.{w_ih,w_hh,b_ih,b_hh}. */
typedef struct pk_lstm_layer {
    pk_tensor w_ih;   /* [4H][in]  gate order i, f, g, o (PyTorch) */
    pk_tensor w_hh;   /* [4H][H]   */
    pk_tensor b_ih;   /* [4H] f32  */
    pk_tensor b_hh;   /* [4H] f32  */
} pk_lstm_layer;

/* Decoder hyper-parameters and weights. Field meaning follows the GGUF metadata
 * parakeet.tdt.* / parakeet.eou.* read at src/parakeet_ctc.cpp:424-460. */
typedef struct pk_model_desc {
    int32_t model_type;            /* PK_MODEL_TDT or PK_MODEL_EOU */
    int32_t d_enc;                 /* encoder d_model (1024 TDT, 512 EOU) */
    int32_t pred_hidden;           /* H: LSTM hidden = embedding dim (640) */
    int32_t joint_hidden;          /* J: joint hidden (640) */
    int32_t n_layers;              /* L: LSTM layers (2 TDT, 1 EOU) */
    int32_t vocab_size;            /* V: joint emits V+1 token logits (blank included) */
    int32_t blank_id;              /* normally V (parakeet_ctc.cpp:430, :454) */
    int32_t num_durations;         /* TDT duration head size (0 for EOU) */
    const int32_t * durations;     /* TDT duration values, num_durations entries */
    int32_t eou_id;                /* EOU <EOU> id (-1: vocab_size-2, parakeet_eou.cpp:182) */
    int32_t eob_id;                /* EOU <EOB> id (-1: vocab_size-1, parakeet_eou.cpp:183) */
    int32_t max_symbols_per_step;  /* default per-frame symbol cap (TDT 10, EOU 5) */
    int32_t n_vocab_pieces;        /* number of tokenizer pieces (EOU special-piece rule) */
    const uint8_t * special_piece; /* EOU: 1 where piece is "<...>" (parakeet_eou.cpp:315-319); may be NULL */
    pk_tensor embed;               /* [V+1][H] predict.embed.weight */
    const pk_lstm_layer * lstm;    /* n_layers entries */
    pk_tensor joint_enc_w;         /* [J][d_enc] */
    pk_tensor joint_enc_b;         /* [J] */
    pk_tensor joint_pred_w;        /* [J][H] */
    pk_tensor joint_pred_b;        /* [J] */
    pk_tensor joint_out_w;         /* [V+1+num_durations][J] */
    pk_tensor joint_out_b;         /* [V+1+num_durations] */
} pk_model_desc;

typedef struct pk_ctx pk_ctx;

/* Math modes for the step loop (pk_set_option(PK_OPT_MATH, ...)). */
enum {
    PK_MATH_F32 = 0,  /* exact dequantized weights, f32 activations, f32 FMA on CUDA cores */
    PK_MATH_TC  = 1,  /* tensor cores (mma.sync f16, f32 accumulate): exact q8_0/f16 weights,
                         activations as f16 hi+lo (22 significant bits); the default when every
                         step-loop weight is q8_0 or f16 and H, J are multiples of 32 */
    PK_MATH_Q8  = 2   /* optional, never the default: the arithmetic of ggml's q8_0 matrix
                         products (vec_dot_q8_0_q8_0), as the reference's graph path runs them:
                         the LSTM, pred-proj and joint-output activations quantised to q8_0 blocks
                         (d = max|x| / 127 per 32 values, q = round(x / d)), one int8 tensor-core
                         product per block scaled by both blocks' d. Persistent loop only (no bulk
                         loop); needs every step-loop weight in q8_0. Logits move by ~1e-2, so
                         tokens differ from the f32 reference at more than its near-ties. */
};

/* Options. */
enum {
    PK_OPT_TIMEOUT_US  = 1,  /* bound (microseconds) on every device-side grid-barrier wait */
    PK_OPT_MATH        = 2,  /* PK_MATH_* */
    PK_OPT_MAX_SYMBOLS = 3,  /* default max_symbols_per_step override (> 0) */
    PK_OPT_TEST_STALL  = 4,  /* test hook: 1 = CTA 0 of the next step loop never arrives at its first
                                grid barrier, so the other CTAs' bounded waits run out and the call
                                returns PK_ERR_TIMEOUT (exercises failure detection without a fault) */
    PK_OPT_BULK_MIN_LIVE = 5, /* tensor-core math: iterations with at least this many live utterances run
                                on the tcgen05 bulk loop (two-dimensional tiles, accumulators in tensor
                                memory), the rest on the persistent loop; default 128, 0 = never,
                                1 = every iteration of a fresh batch (trace runs too) */
    PK_OPT_BULK_SCREEN = 6,  /* bulk-loop iterations with at least this many live utterances (default
                                1024; 0 = never) compute the joint output screened: one f16 product
                                per logit screens the tokens against a proven error bound, and the
                                candidates and the duration logits are recomputed in f32, so the
                                argmax is that of f32 logits; other iterations take three f16
                                products per logit (22-bit activations) and the argmax of those.
                                Trace runs never screen. */
    PK_OPT_BULK_I8 = 7,      /* bulk loop's LSTM and pred-proj GEMMs: 1 (default) = tcgen05 kind::i8 on
                                int16 fixed-point activations and per-row int16-requantised weights, each
                                as two signed int8 digits (three int8 products; the layer-0 input
                                projection from a per-token table); 0 = kind::f16 on f16 hi/lo halves
                                (three f16 products) */
    PK_OPT_BULK_TMA_A = 8    /* bulk loop: 1 (default) = activation rows stored in list order (the joint
                                hidden layer, the pred-proj input, the lower layer's new h) reach shared
                                memory as 2-D TMA boxes and h_prev rows as TMA gather4 loads; 0 = every
                                A row is gathered with cp.async */
};

/* Static information about a context. */
typedef struct pk_info {
    int32_t model_type, d_enc, pred_hidden, joint_hidden, n_layers;
    int32_t vocab_size, blank_id, num_durations, v_plus_1, v_out;
    int32_t eou_id, eob_id, max_symbols_per_step;
    int32_t device, sm_count, grid_ctas;
    uint64_t weight_bytes_device;   /* bytes of repacked weights held on the device */
} pk_info;

/* --- context ------------------------------------------------------------ */

/* Validates the descriptor, dequantizes/repacks every decoder tensor onto
 * `device` and sizes the persistent step-loop kernel. Replaces
 * tdt_prepare_runtime (src/parakeet_tdt.cpp:585) / eou_prepare_runtime
 * (src/parakeet_eou.cpp:172). */
PK_API pk_status pk_create(const pk_model_desc * desc, int device, pk_ctx ** out);
PK_API void      pk_destroy(pk_ctx * ctx);
PK_API pk_status pk_get_info(const pk_ctx * ctx, pk_info * info);
PK_API pk_status pk_set_option(pk_ctx * ctx, int32_t option, int64_t value);
/* Thread-local message describing the last non-OK status of this thread. */
PK_API const char * pk_last_error(void);
PK_API int32_t   pk_abi_version(void);

/* --- batched greedy decode ----------------------------------------------- */

/* A batch of independent utterances (the reference decodes one at a time,
 * src/parakeet_tdt.h:185-205; batching is new here). */
typedef struct pk_batch {
    const float *   enc;               /* f32 [frames][d_enc]; utterance b starts at frame frame_offsets[b] */
    int32_t         enc_on_device;     /* 1: `enc` is a device pointer on the context's device */
    int32_t         B;                 /* number of utterances (>= 0) */
    int32_t         d_enc;             /* must equal the model's d_enc (else PK_ERR_DMODEL) */
    int32_t         max_symbols_per_step; /* <= 0: model default */
    const int64_t * frame_offsets;     /* host, B entries */
    const int32_t * n_frames;          /* host, B entries (>= 0) */
    uint64_t        prefetch_ticket;   /* 0: host input is copied by the call; else a ticket of
                                          pk_prefetch_batch: the call reads that staged copy
                                          (and not `enc`) */
} pk_batch;

/* Results. Pointers are host memory unless results_on_device = 1. Token ids of
 * utterance b are tokens[token_offsets[b] .. token_offsets[b+1]), in emission
 * order (TdtDecodeResult::token_ids, src/parakeet_tdt.h:168-173). */
typedef struct pk_result {
    int32_t   results_on_device;  /* 1: tokens/token_offsets/steps/eou_* are device pointers */
    int32_t * tokens;             /* capacity tokens_cap */
    int64_t   tokens_cap;
    int64_t * token_offsets;      /* B+1 entries */
    int32_t * steps;              /* B entries: joint evaluations (out_steps); may be NULL */
    int32_t * eou_bounds;         /* EOU: segment ends (token index within the utterance); may be NULL */
    int64_t   eou_bounds_cap;
    int64_t * eou_offsets;        /* EOU: B+1 entries into eou_bounds; may be NULL */
    float *   finish_ms;          /* host, B entries: device time from loop start to the utterance's last step; may be NULL */
    /* outputs */
    int64_t   tokens_needed;      /* total tokens emitted (set also on PK_ERR_CAPACITY) */
    int64_t   eou_bounds_needed;
    int64_t   total_steps;        /* sum of steps over the batch */
    int64_t   loop_iterations;    /* batched step-loop iterations */
    int64_t   emit_iterations;    /* iterations in which at least one utterance emitted (LSTM ran) */
    int64_t   kernel_launches;    /* device kernels this call launched */
    double    phase_ms[8];        /* step-loop breakdown seen by CTA 0 (%globaltimer): for the LSTM,
                                     pred/hidden, joint and leader segments, [2i] = CTA 0's own work,
                                     [2i+1] = the rest of the segment (waiting for the slowest CTA
                                     and the grid barrier) */
    double    encproj_ms;         /* device time of the enc-proj GEMM (CUDA events) */
    double    loop_ms;            /* device time of the step loop (bulk and persistent loops together) */
    double    total_ms;           /* device time of the whole call incl. copies */
    double    bulk_ms;            /* device time of the tcgen05 bulk loop (PK_OPT_BULK_MIN_LIVE), 0 if it did not run */
    int64_t   bulk_iterations;    /* loop iterations that ran on the bulk loop (included in loop_iterations) */
    double    bulk_phase_ms[20];  /* bulk loop breakdown seen by CTA 0 (%globaltimer): [0..11] for the LSTM
                                     layers, pred-proj, joint hidden, joint, decision and list
                                     compaction, [2i] = CTA 0's own share, [2i+1] = the grid barrier
                                     after it; [12..19] inside its GEMM phases: A staging waiting for a
                                     free stage, weight loads waiting, MMA issue waiting for A, for the
                                     weights, for a free accumulator, epilogue waiting for an
                                     accumulator, epilogue work, MMA issue */
    int64_t   bulk_steps;         /* joint evaluations made on the bulk loop (of total_steps) */
    int64_t   bulk_lstm_steps;    /* LSTM steps (emissions and initial steps) made on the bulk loop */
    int64_t   bulk_screened_steps;/* of bulk_steps, joint evaluations made screened (PK_OPT_BULK_SCREEN) */
} pk_result;

/* Greedy decode of B fresh utterances (each starts from tdt_init_state /
 * eou_init_state). One persistent kernel runs every step of every utterance
 * on the device; there is no host round trip per token. */
PK_API pk_status pk_decode_batch(pk_ctx * ctx, const pk_batch * batch, pk_result * result);

/* Upper bound on tokens a batch can emit: sum_b n_frames[b] * max(1, max_symbols). */
PK_API int64_t   pk_tokens_capacity(const int32_t * n_frames, int32_t B, int32_t max_symbols_per_step);

/* --- input prefetch (pipelined serving) ----------------------------------- */

/* No counterpart in the reference: its Engine takes one request at a time and
 * has no device copy to overlap (include/parakeet/engine.h:35-55).
 *
 * Starts copying a batch's HOST encoder outputs (frames 0 .. max_b
 * frame_offsets[b] + n_frames[b]) to the device on a copy stream of the context,
 * returns without waiting for the copy, and writes a ticket (nonzero) naming the
 * staged copy to *ticket. A decode call (pk_decode_batch, pk_decode_trace) whose
 * pk_batch carries that ticket in prefetch_ticket reads the staged copy -- the
 * device waits for it -- instead of copying `enc`; the batch must not read more
 * frames than the prefetch covered. A ticket is used once. At most two copies are
 * staged: a prefetch made while two are staged replaces the older one, and its
 * ticket is no longer valid. A decode given a ticket that is not staged (used
 * already, replaced) or that covers too few frames fails with PK_ERR_INVALID and
 * copies nothing. Calls without a ticket (prefetch_ticket = 0, device input,
 * pk_stream_window) leave the staged copies alone. So the copy of batch k+1
 * overlaps the decode of batch k:
 *
 *     pk_prefetch_batch(ctx, &b[0], &b[0].prefetch_ticket);
 *     for (k = 0; k < n; ++k) {
 *         if (k + 1 < n) pk_prefetch_batch(ctx, &b[k + 1], &b[k + 1].prefetch_ticket);
 *         pk_decode_batch(ctx, &b[k], &res[k]);
 *     }
 *
 * The staged copy is the host buffer as it was when the copy ran: the buffer
 * must stay valid and unchanged until the copy has completed, which is when the
 * decode that uses the ticket returns, or the second later pk_prefetch_batch call
 * returns, whichever comes first; after that the caller may refill it. Pinned
 * host memory makes the copy asynchronous; pageable memory is copied before this
 * call returns. A batch with enc_on_device = 1 is rejected (PK_ERR_INVALID); a
 * batch that reads no frames stages nothing and gets ticket 0. The decode's
 * total_ms does not include a prefetched copy except for any wait for it. */
PK_API pk_status pk_prefetch_batch(pk_ctx * ctx, const pk_batch * batch, uint64_t * ticket);

/* --- teacher-forced trace (parity harness) -------------------------------- */

/* Runs the same kernel as pk_decode_batch but, when forced_token is given,
 * replaces the device argmax of step s of utterance b with the caller's
 * decision (forced_token / forced_dur_idx, [B][max_steps]; a negative token
 * means "use the device argmax") so the device follows the oracle's
 * trajectory. Records per step: logits [B][max_steps][v_out], the device's own
 * argmax, and the LSTM state after the step [B][max_steps][L][H]. */
typedef struct pk_trace {
    int32_t         max_steps;
    const int32_t * forced_token;     /* host [B][max_steps] or NULL (free running) */
    const int32_t * forced_dur_idx;   /* host [B][max_steps] or NULL */
    float *         logits;           /* host [B][max_steps][v_out] or NULL */
    float *         h;                /* host [B][max_steps][L][H] or NULL */
    float *         c;                /* host [B][max_steps][L][H] or NULL */
    int32_t *       argmax_token;     /* host [B][max_steps] or NULL */
    int32_t *       argmax_dur_idx;   /* host [B][max_steps] or NULL */
} pk_trace;

PK_API pk_status pk_decode_trace(pk_ctx * ctx, const pk_batch * batch, pk_trace * trace, pk_result * result);

/* --- streaming (tdt_decode_window / eou_decode_window) -------------------- */

/* Per-utterance decoder state (TdtDecodeState, src/parakeet_tdt.h:175-183;
 * EouDecodeState, src/parakeet_eou.h:53-66), kept on the device. */
typedef struct pk_stream pk_stream;

/* Host view of a stream's state, for export / import (resume). */
typedef struct pk_stream_state {
    float * h;                    /* [L][H] */
    float * c;                    /* [L][H] */
    float * pred_out;             /* [H] last-layer h (the prediction-net output) */
    int32_t symbols_this_step;
    int32_t carry_frames;         /* TDT: frames the last duration jumped past the window */
    int32_t initialized;
    int32_t last_token;           /* EOU */
    int32_t segment_start_token;  /* EOU */
} pk_stream_state;

PK_API pk_status pk_stream_create(pk_ctx * ctx, pk_stream ** out);
PK_API void      pk_stream_destroy(pk_stream * s);
/* tdt_init_state / eou_init_state: h = c = 0, one LSTM step on embed[blank]. */
PK_API pk_status pk_stream_reset(pk_stream * s);
/* Decode one window of n_frames encoder frames, continuing the stream's state.
 * `n_tokens_before` is the caller's running token count on entry (the size of
 * out_tokens in the reference); EOU boundaries are expressed in that count.
 * tokens receives only this window's tokens. Mirrors tdt_decode_window's
 * semantics: n_frames <= 0 returns 0 without initialising (TDT); an
 * uninitialised state is initialised first; carry_frames crosses windows. */
PK_API pk_status pk_stream_window(pk_stream * s, const float * enc, int32_t enc_on_device,
                           int32_t n_frames, int32_t d_enc, int32_t max_symbols_per_step,
                           int32_t n_tokens_before,
                           int32_t * tokens, int32_t tokens_cap, int32_t * n_tokens,
                           int32_t * steps,
                           int32_t * eou_bounds, int32_t bounds_cap, int32_t * n_bounds);
PK_API pk_status pk_stream_get_state(const pk_stream * s, pk_stream_state * st);
PK_API pk_status pk_stream_set_state(pk_stream * s, const pk_stream_state * st);

/* --- multi-GPU host helper ------------------------------------------------ */

/* Longest-processing-time partition of utterances over n_shards devices by
 * frame count (descending T, each to the shard with the least total T; ties
 * to the lowest shard id). shard_of[b] receives the shard of utterance b. */
PK_API pk_status pk_shard_lpt(const int32_t * n_frames, int32_t B, int32_t n_shards, int32_t * shard_of);

/* Partition that balances each shard's modelled decode time rather than its
 * frames (no counterpart in the reference, which decodes on one device). A call
 * lasts as long as its longest utterance's sequential decode, and one loop
 * iteration costs little more with a few more utterances live, so long utterances
 * are best decoded together on a shard rather than each setting its own shard's
 * time. Model: decode steps proportional to frames, one iteration's cost a
 * piecewise-linear function of the live count measured on B200 (persistent loop
 * below 128 live, bulk loop from 128). First fit decreasing (descending frame
 * count, each utterance to the lowest shard whose modelled time stays within a
 * bound) with the bound bisected to the smallest that places every utterance.
 * Shards may differ widely in size. Deterministic: every rank computes the same
 * partition. */
PK_API pk_status pk_shard_balanced(const int32_t * n_frames, int32_t B, int32_t n_shards, int32_t * shard_of);

/* --- decode without device allocation ------------------------------------- */

/* No counterpart in the reference. Greedy decode of ONE fresh utterance that
 * allocates no device memory during the call. For callers that cannot call
 * cudaMalloc while decoding: a process running under a fixed device-memory
 * budget whose allocator forbids new allocations after start-up, or a
 * latency-critical audio thread where cudaMalloc's implicit device
 * synchronisation and possible failure are not acceptable.
 *
 * Every buffer the decode needs beyond its inputs and outputs lives in one
 * statically sized device array inside the library (PK_NOALLOC_SCRATCH_BYTES,
 * held by every GPU that loads the library until the process exits). Limits:
 * n_frames <= PK_NOALLOC_MAX_FRAMES, joint_hidden and pred_hidden <= 1024.
 * Larger inputs are rejected with PK_ERR_INVALID. The context (weights) must
 * already exist (pk_create allocates; this call does not).
 *
 * enc, tokens, n_tokens and steps are DEVICE pointers on the context's device;
 * tokens_cap must be >= n_frames * max(1, max_symbols_per_step). On success
 * *n_tokens and *steps (device int32) hold the token count and joint
 * evaluations (tdt_greedy_decode / eou_greedy_decode semantics for one
 * utterance). The input must be written and the outputs free before the call:
 * the decode runs on the context's own stream, which does not wait for work
 * the caller queued on other streams.
 *
 * It always runs the f32 CUDA-core enc-proj and step loop (PK_MATH_F32),
 * whatever the context's math mode, so its tokens equal pk_decode_batch's
 * with math = PK_MATH_F32. pk_create has already looked up the array's device
 * address (cudaGetSymbolAddress), which loads the array with the library's
 * module when CUDA loads modules lazily, and has run one decode on that loop,
 * so a call made right after pk_create allocates nothing. All calls share the
 * one array, which keeps the last call's contents: calls that overlap on the
 * GPU (from several threads or contexts on the same device) race with each
 * other and must be serialised by the caller. The call blocks until its
 * decode has finished and leaves the caller's current device as it was. */
#define PK_NOALLOC_MAX_FRAMES 4096
#define PK_NOALLOC_SCRATCH_BYTES (17u * 1024u * 1024u)
PK_API pk_status pk_decode_noalloc(pk_ctx * ctx, const float * enc, int32_t n_frames, int32_t d_enc,
                                   int32_t max_symbols_per_step, int32_t * tokens, int32_t tokens_cap,
                                   int32_t * n_tokens, int32_t * steps);

/* ---- Beside the token loop: CTC greedy decode and detokenize -----------------
 *
 * Both work on B utterances at once on one device. Host arrays are plain
 * pointers; a `*_on_device` flag says whether the large input (logits,
 * tokens) is a device pointer on the handle's device (4-byte aligned) or host
 * memory. Outputs are written to host memory. */

typedef struct pk_ctc pk_ctc;

/* Replaces the per-utterance calls of ctc_greedy_decode / ctc_greedy_decode_window
 * (src/parakeet_ctc.cpp:1820-1865, called at src/parakeet_engine.cpp:299 and
 * src/main.cpp:777). vocab_size = logits row width (tokens + blank). */
PK_API pk_status pk_ctc_create(int device, int32_t vocab_size, int32_t blank_id, pk_ctc ** out);
PK_API void      pk_ctc_destroy(pk_ctc * c);

/* logits: [sum n_frames][vocab_size] f32, utterance b at rows frame_offsets[b] ..
 * frame_offsets[b] + n_frames[b] - 1. Each frame's argmax is the first index of
 * its maximum (`>` scan from index 0, so a NaN at index 0 wins and other NaNs
 * never do); a frame emits its argmax when it is not blank and differs from the
 * previous frame's argmax. prev_inout[b] (host) is the argmax of the frame
 * before the window (-1 for a fresh utterance) and receives the window's last
 * argmax (ctc_greedy_decode_window's inout_prev_token). tokens (host, tokens_cap
 * entries) receive the emitted tokens of all utterances back to back,
 * token_offsets (host, B + 1) their start indices, first_frame (host, may be
 * NULL) each token's frame index within its utterance's window. tokens_needed
 * (host, may be NULL) receives the total; PK_ERR_CAPACITY when it exceeds
 * tokens_cap (prev_inout is then left unchanged). */
PK_API pk_status pk_ctc_greedy(pk_ctc * c, const float * logits, int32_t logits_on_device,
                               const int64_t * frame_offsets, const int32_t * n_frames, int32_t B,
                               int32_t * prev_inout, int32_t * tokens, int64_t tokens_cap,
                               int64_t * token_offsets, int32_t * first_frame, int64_t * tokens_needed);

typedef struct pk_vocab pk_vocab;

/* Replaces parakeet::detokenize (src/sentencepiece_bpe.cpp:9-37) with its
 * BpeVocab (src/sentencepiece_bpe.h): piece v is the byte string
 * piece_bytes[piece_offsets[v] .. piece_offsets[v + 1]) (UTF-8, as the GGUF
 * tokenizer stores it). blank / bos / eos / pad ids (-1: none) are skipped. */
PK_API pk_status pk_vocab_create(int device, const uint8_t * piece_bytes, const int64_t * piece_offsets,
                                 int32_t n_pieces, int32_t blank_id, int32_t bos_id, int32_t eos_id,
                                 int32_t pad_id, pk_vocab ** out);
PK_API void      pk_vocab_destroy(pk_vocab * v);

/* tokens: [token_offsets[B]] int32 (host, or device when tokens_on_device),
 * utterance b = tokens[token_offsets[b] .. token_offsets[b + 1]) (token_offsets
 * on the host). Ids outside [0, n_pieces) and the special ids are skipped; each
 * U+2581 (E2 96 81) inside a piece becomes one space; leading spaces of each
 * utterance's text are removed. text (host, text_cap bytes) receives the B
 * texts back to back (no terminators), text_offsets (host, B + 1) their start
 * offsets, text_needed (host, may be NULL) the total; PK_ERR_CAPACITY when it
 * exceeds text_cap. */
PK_API pk_status pk_detokenize(pk_vocab * v, const int32_t * tokens, int32_t tokens_on_device,
                               const int64_t * token_offsets, int32_t B, char * text, int64_t text_cap,
                               int64_t * text_offsets, int64_t * text_needed);

#ifdef __cplusplus
}
#endif

#endif /* PARAKEET_CUDA_H */
