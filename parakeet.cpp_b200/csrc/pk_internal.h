// pk_internal.h -- host/device declarations shared by libparakeet_cuda's
// translation units (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "parakeet_cuda.h"

namespace pk {

constexpr int kMaxLayers = 4;
constexpr int kThreads = 256;      // step-loop CTA size (8 warps)
constexpr int kWarps = kThreads / 32;

// Per-utterance integer state, [B][kUst] in device memory.
enum UstField : int {
    U_T = 0,          // current frame index t (frame pointer)
    U_SYM,            // symbols_this_step (working value)
    U_NTOK,           // tokens emitted in this call
    U_STEPS,          // joint evaluations in this call (out_steps)
    U_HBUF,           // which of the two h buffers holds the current state
    U_LAST,           // EOU last_token
    U_SEGSTART,       // EOU segment_start_token (in the caller's running count)
    U_NBND,           // EOU boundaries recorded in this call
    U_NBEFORE,        // caller's running token count on entry (EOU boundary base)
    U_NFRAMES,        // window length T
    U_SYMX,           // EOU symbols_this_step as left by the last finished frame
    kUst = 16
};

// Control words, int32 [kCtl] in device memory.
enum CtlField : int {
    C_ERR = 0,        // pk_status set by the device (timeout / index check)
    C_SEL,            // which live list is current
    C_NLIVE0,         // live count of list 0
    C_NLIVE1,         // live count of list 1
    C_NEMIT,          // entries in the emit list
    C_NDECIDED,       // utterances decided by the last leader (trace bookkeeping)
    C_ITERS,          // batched loop iterations completed
    C_ERRINFO,        // first failing utterance / index (diagnostics)
    C_EMITITERS,      // iterations whose leader produced a non-empty emit list
    C_BULKITERS,      // iterations run by the bulk loop (pk_bulk.cu) before the persistent loop
    C_BULKSTEPS,      // joint evaluations (live utterance-iterations) on the bulk loop
    C_BULKEMITS,      // LSTM steps (emit-list entries) on the bulk loop
    C_BULKSCREENED,   // joint evaluations of the bulk loop made screened (one f16 product)
    kCtl = 16
};

constexpr int kTcM = 16;         // utterances per tensor-core pass (mma M)
constexpr int kTcRmax = 8;       // 8-row weight tiles per tensor-core GEMM group
constexpr int kTcRec = 256;     // records staged in shared memory per block of a phase

// One phase's weights in the tensor-core layout. Rows owned by CTA k are
// padded to `tiles` tiles of 8 rows; per (tile, 32-wide K block, lane) the
// lane's B fragments of mma.m16n8k16 for the block's two k-steps are stored
// contiguously: q8_0 as biased bytes (q + 128, 8 B per lane) with an f32 scale
// per (tile, block, row); f16 weights as halves (16 B per lane).
struct TcBlock {
    const uint8_t * frag;      // global [grid][cta_bytes]
    const float * scale;       // global [grid][cta_scales] (q8_0 only)
    unsigned cta_bytes;
    unsigned cta_scales;       // floats per CTA
    int tiles;
    int K;                     // multiple of 32
    int is_i8;
    int imma;                  // q8_0 packed as raw int8 B fragments of mma.m16n8k32 (int16 activations)
    unsigned sm_frag;          // offsets inside the stationary shared-memory region
    unsigned sm_scale;
};

// Everything the persistent step-loop kernel needs (passed by value).
struct LoopParams {
    // geometry
    int H, J, L, V1, Vo, Nd, blank, eou, eob, is_tdt, max_sym, B, n_special;
    int chunk;                 // max utterances per shared-memory chunk (power of two, <= 32)
    int ldx;                   // floats per chunk row in shared memory (>= max(2H, J))
    long long timeout_ns;      // bound on every grid-barrier wait
    int max_iters;             // bound on batched loop iterations (max_b T_b * (max_sym + 1) + 2)
    int test_stall;            // test hook: CTA 0 returns before its first barrier
    int resume;                // the loop continues a batch that the bulk loop (pk_bulk.cu) started:
                               // control words, lists and state come from it, iteration counts add on
    // tensor-core phases (tc = 1)
    int tc;
    int stationary;            // copy TC weights into shared memory at kernel start
    unsigned sm_weights;       // bytes of the stationary region
    int rbh, rbj;              // bytes per staged row: h (2 H es + 16), hid (4 J + 16)
    int area;                  // bytes of the shared-memory staging area (multiple of 16)
    int mb;                    // m16 blocks per pass: passes of 16 * mb utterances
    int rpc_j, rpc_p, upc;     // joint rows, pred rows, LSTM units per CTA
    int h_int;                 // LSTM outputs staged as int16 fixed point (two int8 digit planes)
    int q8;                    // PK_MATH_Q8: staged activations quantised to q8_0 blocks, int8 products
    TcBlock tcj, tcp, tcl[kMaxLayers];
    const float * g0;          // [V+1][4H]: b_ih0 + W_ih0 . embed[v] (layer-0 input projection)
    // weights (f32, row-major [out][in])
    const float * embed;
    const float * w_ih[kMaxLayers];
    const float * w_hh[kMaxLayers];
    const float * b_ih[kMaxLayers];
    const float * b_hh[kMaxLayers];
    const float * pred_w;
    const float * pred_b;
    const float * out_w;
    const float * out_b;
    const int32_t * durations;
    const uint8_t * special;
    // inputs
    const float * encp;        // [frames][J] enc-proj incl. bias
    const int64_t * frame_off; // [B]
    // state
    float * h;                 // [2][L][B][H]
    float * c;                 // [L][B][H]
    float * predp;             // [B][J]
    float * hid;               // [B][J] (CUDA-core phases)
    // tensor-core phases: activation rows in the staged layout [hi part | lo part | pad]
    // (h: int16 digit planes of 1 byte or f16 halves, es bytes each; hid: f16)
    unsigned char * hst;       // [2][L][B] rows of rbh bytes: h state per (buffer, layer, utterance)
    unsigned char * xnew;      // [L][B] rows of rbh bytes: new h by emit-list index
    unsigned char * hidc;      // [B] rows of rbj bytes: joint hidden by live-list index
    int32_t * ust;             // [B][kUst]
    unsigned long long * keys; // [2][B][2] packed argmax keys (token, duration), buffer = iteration & 1
    int32_t * live;            // [2][B]
    int64_t * live_frame;      // [2][B] encoder row (frame_offset + t) of each live entry
    int32_t * emit;            // [B][2]: utterance, token | h-buffer << 30 | reset << 31
    int32_t * ctl;             // [kCtl]
    unsigned int * bar;        // [8]: counter-barrier arrivals, -, leader arrivals, -, 64-bit release word, -
    unsigned long long * t_start;   // [1] globaltimer at loop start
    unsigned long long * prof;      // [8] CTA 0 phase breakdown (ns), see pk_result::phase_ms
    unsigned long long * finish_ns; // [B]
    // outputs
    int32_t * tok_out;         // per-utterance regions
    const int64_t * tok_region;// [B] region start
    int32_t * bnd_out;         // EOU boundaries, per-utterance regions (cap T)
    const int64_t * bnd_region;
    // teacher-forced trace (trace_steps == 0: off)
    int trace_steps;
    const int32_t * forced_tok;
    const int32_t * forced_dur;
    float * tr_logits;         // [B][S][Vo]
    float * tr_h;              // [B][S][L][H]
    float * tr_c;
    int32_t * tr_tok;
    int32_t * tr_dur;
};

// ---- bulk loop (pk_bulk.cu): iterations with many live utterances on tcgen05 ----
//
// One weight matrix of a step-loop GEMM, split into exact f16 halves (w = hi + lo)
// for the tensor-memory loop: [N][K] f16 each, TMA descriptors (128 bytes each,
// 64-byte aligned, in device memory) with a 64 x 64 box and 128-byte swizzle.
struct BulkGemm {
    const void * map_hi;
    const void * map_lo;
    const void * hi;           // the f16 halves themselves, [N][K] each (hi + lo = the weight, exactly)
    const void * lo;
    int N, K;
    int i8;                    // int8 digit planes instead of f16 halves: each row requantised to int16,
                               // W = 256 hi + lo with hi, lo signed bytes, weight = W * rscale[row]
    const float * rscale;      // [N] (i8)
    int lo_zero;               // every lo half is zero (f16 weights): two products, no lo tiles
};

struct BulkParams {
    LoopParams P;              // lists, state, outputs and control words shared with the persistent loop
    int min_live;              // iterate while at least this many utterances are live
    BulkGemm gl[kMaxLayers];   // LSTM layer l: rows 4j + q = gate q of unit j; K = [W_ih | W_hh]
    BulkGemm gp;               // joint.pred [J][H]
    BulkGemm gj;               // joint.out [Vo][J]
    const float * lbias;       // [L][4H] gate biases b_ih + b_hh in the same row order
    const unsigned char * e16; // [V+1] rows of 4H bytes: f16 hi | lo of the embedding (layer 0's x)
    const float * g0b;         // [V+1][4H] (int8 LSTM): b_ih0 + b_hh0 + W_ih0 . embed[v], rows 4j + q
    unsigned char * h16;       // [2][L][B] rows of 4H bytes: f16 hi[H] | lo[H] of h, by utterance
    unsigned char * x16;       // [L][B] rows, same layout: layer l's new h by emit-list index
    int2 * dcount;             // [grid] each CTA's (emit, live) counts from the decision
    unsigned long long * prof; // [20] CTA 0: time per phase and per GEMM role (ns), see pk_result::bulk_phase_ms
    // Screened joint (iterations with at least screen_min live utterances; 0 = never):
    // the joint GEMM takes one f16 product (A_hi W_hi) and keeps, per (live row, N
    // tile), its four largest token logits; the decision recomputes in f32 every token
    // whose approximate logit is within twice a proven error bound of the row's
    // maximum, and every duration logit.
    // 2-D TMA descriptors (CUtensorMap, 128 bytes) of the compact activation rows, bytes as
    // elements, 128 x 128-byte boxes, 128-byte swizzle: x16 ([L][B] rows of 4H bytes) and hidc
    // ([B] rows of rbj bytes); tma_a = 0 stages every A row with cp.async instead
    alignas(64) unsigned char map_x16[128];
    alignas(64) unsigned char map_hid[128];
    // the h state rows ([2][L][B] rows of 4H bytes, then one zero row) with 1-row boxes for
    // tile::gather4: h_prev rows, indexed by utterance, four rows per TMA instruction
    alignas(64) unsigned char map_h16[128];
    int h16_zero_row;
    int tma_a;
    int screen_min;
    float * norm2;             // [B] sum of squares of the joint hidden row, by live index
    uint4 * jsum;              // [B][jsum_stride][2] per (live row, N tile): (m1..m4 bits), (j1, j2, j3, NaN flag)
    int jsum_stride;           // N tiles of the narrowest joint tiling: ceil(Vo / 64)
    int n_scr;                 // token rows [0, n_scr) screened (a multiple of 64); rows [n_scr, V1) and the
                               // duration rows are always recomputed in f32
    const float * wnorm;       // device: max over token rows of joint.out of ||row||_2 (rounded up)
};

// Device-side bulk weights of a context (built once at pk_create).
struct BulkWeights {
    void * mem = nullptr;      // one allocation: f16 halves, biases, TMA descriptors
    BulkGemm gl[kMaxLayers]{}, gp{}, gj{};
    BulkGemm gli[kMaxLayers]{}, gpi{};   // the LSTM and pred-proj matrices as int8 digit planes (i8 = 1);
                                         // layer 0 without W_ih (its input projection is g0b)
    int i8_ok = 0;
    const float * lbias = nullptr;
    const unsigned char * e16 = nullptr;
    const float * g0b = nullptr;
    const float * wnorm = nullptr;   // max row norm of joint.out's token rows (screened joint)
    size_t bytes = 0;
};
bool        bulk_supported(int H, int J, int L);
bool        bulk_screen_supported(int J);
cudaError_t bulk_row_map(void * map, const void * base, long long rows, long long row_bytes);
cudaError_t bulk_row_map_gather(void * map, const void * base, long long rows, long long row_bytes);   // the screened joint's row norms need J % 128 == 0
cudaError_t bulk_prepare(BulkWeights & w, int H, int J, int L, int Vo, int V1, const float * embed,
                         const float * const * w_ih, const float * const * w_hh, const float * const * b_ih,
                         const float * const * b_hh, const float * pred_w, const float * out_w,
                         const int * f16_weights, const float * g0, cudaStream_t s);
void        bulk_release(BulkWeights & w);
size_t      bulk_smem_bytes();
cudaError_t bulk_configure();
cudaError_t bulk_occupancy(int * blocks_per_sm);
int         bulk_threads();
cudaError_t launch_bulk(const BulkParams & q, int grid, cudaStream_t s);

// Launch wrappers (defined in the .cu files).
cudaError_t launch_step_loop(const LoopParams & p, int grid, size_t smem, cudaStream_t s);
size_t      step_loop_smem_bytes(int chunk, int ldx, int H, int grid);
size_t      step_loop_tc_smem_bytes(unsigned sm_weights, int area, int rpc_j, int rpc_p, int upc);
cudaError_t step_loop_configure(size_t smem, int tc);
size_t step_loop_static_smem(int tc);   // static shared memory of the step-loop kernel
cudaError_t step_loop_occupancy(size_t smem, int tc, int * blocks_per_sm);

cudaError_t launch_encproj_f32(const float * enc, int64_t frames, int De, const float * w,
                               const float * b, int J, float * out, cudaStream_t s);

cudaError_t launch_dequant(const void * src, int type, int64_t ne0, int64_t rows,
                           float * dst, cudaStream_t s);

// offsets[b+1] = offsets[b] + ust[b][field].
cudaError_t launch_scan(const int32_t * ust, int B, int field, int64_t * offsets, cudaStream_t s);
// Copy each utterance's region src[region[b] ...] to dst[offsets[b] ...].
cudaError_t launch_gather(const int32_t * ust, int B, int field, const int32_t * src,
                          const int64_t * region, const int64_t * offsets, int32_t * dst,
                          cudaStream_t s);
// hi = f16(x), lo = f16(x - hi) for n floats.
// x -> round(x * 2^15) clamped to +-32767, stored as two int8 digit planes
// (hi = value >> 8 signed, lo = value & 255 unsigned).
cudaError_t launch_split_int16(const float * src, unsigned char * hi, unsigned char * lo, int64_t n, cudaStream_t s);
// rows of H values (n_rows of them) -> staged-layout rows of rb bytes (hi part then
// lo part): int16 digits (es = 1) or f16 halves (es = 2).
cudaError_t launch_stage_rows(const float * src, int n_rows, int H, int es, int rb, unsigned char * dst,
                              cudaStream_t s);
cudaError_t launch_split_f16(const float * src, unsigned short * hi, unsigned short * lo, int64_t n,
                             cudaStream_t s);
// Tensor-core joint.enc projection (pk_encproj.cu): weights split into f16 hi / lo
// halves once ([2J][K] f16 in w16, TMA descriptor of 128 bytes in tmap_out).
bool        encproj_tc_supported(int K, int J);
size_t      encproj_tc_smem_bytes();
cudaError_t encproj_tc_configure();
cudaError_t encproj_tc_prepare(const float * w, int J, int K, unsigned short * w16, void * tmap_out,
                               cudaStream_t s);
cudaError_t launch_encproj_tc(const float * enc, long long frames, int K, const void * tmap, int J,
                              const float * bias, float * out, long long timeout_ns, int * err, cudaStream_t s);
// Up to 12 copies from pinned host memory (device-readable) to device memory, in one
// kernel; sizes are multiples of 4 bytes, addresses 4-byte aligned.
struct HostSegment {
    const void * src;
    void * dst;
    unsigned long long bytes;
};
struct HostSegments {
    HostSegment seg[12];
    int n;
};
cudaError_t launch_copy_segments(const HostSegments & g, cudaStream_t s);
cudaError_t launch_extract_field(const int32_t * ust, int B, int field, int32_t * dst,
                                 cudaStream_t s);

// Read-only view of a context for entry points defined outside pk_api.cu.
struct CtxView {
    int device, grid, chunk, ldx;
    size_t smem;
    cudaStream_t stream;
    int H, J, De, L, V1, Vo, Nd, blank, eou, eob, is_tdt, max_sym, n_special;
    long long timeout_ns;
    const float * embed;
    const float * w_ih[kMaxLayers];
    const float * w_hh[kMaxLayers];
    const float * b_ih[kMaxLayers];
    const float * b_hh[kMaxLayers];
    const float * enc_w;
    const float * enc_b;
    const float * pred_w;
    const float * pred_b;
    const float * out_w;
    const float * out_b;
    const int32_t * durations;
    const uint8_t * special;
};
void ctx_view(const pk_ctx * ctx, CtxView * v);
// pk_noalloc.cu: loads the no-allocation path's module on `device` (current).
pk_status noalloc_prepare(int device);
// Records `msg` as this thread's pk_last_error() text and returns s.
pk_status set_error(pk_status s, const char * msg);

}  // namespace pk
