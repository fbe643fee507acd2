// pk_bulk.cu -- the greedy step loop for iterations with many live utterances,
// on the 5th-generation tensor cores (tcgen05.mma, accumulators in tensor memory).
//
// The persistent loop (pk_loop.cu) keeps every weight slice stationary in one
// CTA's shared memory, so each CTA reads every live utterance's activation row
// once per phase: with thousands of live utterances that is 148 reads of each
// row per iteration, and the loop is bound by L2 ingress rather than by the
// tensor cores. This loop instead tiles every step-loop GEMM in two dimensions,
//
//   tile = 128 utterances (UMMA M) x up to 256 weight rows (UMMA N), K in steps of 64,
//
// streaming both operands from L2 (the weights, ~42 MB as f16 halves, stay
// L2-resident), so an activation row is read once per weight tile and a weight
// tile once per utterance tile. It runs while at least `min_live` utterances are
// live and then exits; the persistent loop continues the same batch from the
// state, lists and control words left here (LoopParams::resume).
//
// Per iteration (same order and semantics as the persistent loop):
//   LSTM layer l   gates[e] = W_ih x + W_hh h_prev for the emit list (x = the token's
//                  embedding row for layer 0, the new h of layer l-1 above), then the
//                  cell update with b_ih + b_hh in the epilogue (host_lstm_step,
//                  src/parakeet_tdt.cpp:106-142)
//   pred           predp[utt] = b_pred + W_pred h[L-1] for the emit list
//   hidden         hidc[i] = relu(encp[t_i] + predp[utt_i]) for the live list
//                  (host_joint_step, :154-177)
//   joint          logits = b_out + W_out hid, folded into 64-bit argmax keys
//                  (argmax_f32, :25-32: first index of the maximum)
//   decision       the greedy control (tdt_decode_window :938-968, eou_decode_window
//                  src/parakeet_eou.cpp:271-333) for a slice of the live list per
//                  CTA, then the next emit and live lists compacted over all CTAs
// separated by grid barriers (bounded waits, like every wait here).
//
// Arithmetic: both operands as exact-or-22-bit f16 halves, three products
// (A_hi W_hi + A_lo W_hi + A_hi W_lo) accumulated in f32 in tensor memory: the
// weights' halves are exact for q8_0 (d * q has at most 18 significant bits) and
// f16; h and the joint hidden layer carry 22 significant bits; the dropped
// A_lo W_lo term is ~2^-22 relative.
//
// Warp roles in a GEMM phase (12 warps): 0-3 stage A (one utterance row per
// thread, 16-byte cp.async gathers into the 128-byte-swizzled K-major tile), 4
// issues the weight tiles' TMA loads, 5 owns tensor memory and issues the MMAs
// (two 256-column accumulators: the epilogue of one tile overlaps the next tile's
// main loop), 8-11 run the epilogue (TMEM lane quarter = warp % 4). All warps
// run the element-wise and decision phases.

#include "pk_device.cuh"
#include "pk_umma.cuh"

#include <vector>

namespace pk {
namespace {

constexpr int kBThreads = 384;
constexpr int kBWarps = kBThreads / 32;
constexpr int kBM = 128;                              // utterances per tile (UMMA M)
constexpr int kBK = 64;                               // K per stage: one 128-byte f16 row
constexpr int kBNmax = 256;                           // weight rows per tile (UMMA N)
constexpr int kMaxStages = 4;
constexpr unsigned kATile = kBM * kBK * 2;            // one f16 plane of an A stage (16 KB)
constexpr unsigned kBBox = 64 * kBK * 2;              // one 64-row box of one B plane (8 KB)
constexpr unsigned kRing = 192 * 1024;                // operand ring: 2 stages at N = 256, 3 at 128, 4 at 64
constexpr unsigned kTmemCols = 2 * kBNmax;            // two accumulators

struct BulkSmem {
    unsigned long long full_a[kMaxStages];
    unsigned long long full_b[kMaxStages];
    unsigned long long empty[kMaxStages];
    unsigned long long acc_full[2];
    unsigned long long acc_empty[2];
    const unsigned char * a_s0[kBM];   // A rows of the current tile: segment-0 source
    const unsigned char * a_s1[kBM];   // segment-1 source
    int a_r1[kBM];                     // segment-1 row of the h16 map (h_prev; the zero row for resets)
    unsigned char a_fl[kBM];           // bit 0: row in the batch, bit 1: segment 1 is zero
    unsigned long long rprof[8];       // CTA 0, per role: waits and work inside the GEMM phases (ns)
    int tok_s[kBThreads];              // screened joint: this CTA's slice of the live list, exact argmax
    int dur_s[kBThreads];
    unsigned tmem_base;
    int err;                       // a wait of this CTA gave up (shared by every role)
    int scan[kBWarps + 2];
    int flag[4];
};

enum { G_LSTM = 0, G_PRED = 1, G_JOINT = 2 };

// Uses of every ring slot and accumulator so far: each role advances its own, in the
// same order, so the mbarrier phase of a slot is its use count's parity. (The number
// of slots changes with the tile width from phase to phase; every slot is drained at
// the end of a phase.)
struct Pipe {
    unsigned ua[kMaxStages] = {0u, 0u, 0u, 0u};   // A stages filled
    unsigned ub[kMaxStages] = {0u, 0u, 0u, 0u};   // B stages filled
    unsigned um[kMaxStages] = {0u, 0u, 0u, 0u};   // stages consumed by the MMAs
    unsigned acc_m = 0, acc_e = 0;                // tiles accumulated (MMA) / drained (epilogue)
};

// Ring geometry of a phase: a stage is the A tile (hi[, lo]) then the B tile (hi[, lo])
// of bn rows; every part starts on a 1024-byte boundary (the swizzle atom). The
// screened joint keeps only the hi planes (planes = 1).
struct Ring {
    unsigned stage, b_plane, b_off;
    int n;
};
__device__ __forceinline__ Ring ring(int bn, int planes) {
    Ring r;
    r.b_plane = (unsigned) bn * kBK * 2u;
    r.b_off = (unsigned) planes * kATile;
    r.stage = r.b_off + (unsigned) planes * r.b_plane;
    r.n = min(kMaxStages, (int) (kRing / r.stage));
    return r;
}

struct Job {
    int kind, l, M, N, nK, bn, nM, nN, tiles, split, sel, planes;
    int kel;                   // K elements per stage (one 128-byte row per plane): 64 f16, 128 int8
    const BulkGemm * g;
};

// Iterations whose joint runs screened (one product, exact recomputation of the candidates).
__device__ __forceinline__ bool screened(const BulkParams & Q, int n_live) {
    return Q.screen_min > 0 && n_live >= Q.screen_min;
}

__device__ __forceinline__ Job make_job(const BulkParams & Q, int kind, int l, int M, int sel) {
    Job j{};
    j.kind = kind;
    j.l = l;
    j.M = M;
    j.sel = sel;
    j.g = kind == G_LSTM ? &Q.gl[l] : kind == G_PRED ? &Q.gp : &Q.gj;
    // the screened joint covers the token rows [0, n_scr) only (the last few token rows
    // and the duration rows are recomputed exactly by the decision)
    j.N = (kind == G_JOINT && screened(Q, M)) ? Q.n_scr : j.g->N;
    j.kel = j.g->i8 ? 2 * kBK : kBK;
    j.nK = j.g->K / j.kel;
    j.nM = (M + kBM - 1) / kBM;
    // LSTM: K = [x | h_prev] (int8 layer 0: h_prev only, its input projection is a table)
    j.split = kind == G_LSTM ? ((j.g->i8 && l == 0) ? 0 : Q.P.H / j.kel) : 0;
    j.planes = (kind == G_JOINT && screened(Q, M)) ? 1 : 2;
    // tile width: fewest rounds of tiles over the CTAs, counting ~32 columns of
    // fixed cost per tile (pipeline fill and drain); int8 tiles hold two accumulators
    // (the 2^16 and 2^8 digit levels) per buffer, so at most 128 columns
    const int G = (int) gridDim.x;
    const int bnmax = j.g->i8 ? kBNmax / 2 : kBNmax;
    int best = bnmax;
    long long best_cost = -1;
    for (int bn = bnmax; bn >= 64; bn >>= 1) {
        const long long tiles = (long long) j.nM * ((j.N + bn - 1) / bn);
        const long long cost = ((tiles + G - 1) / G) * (bn + 32);
        if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = bn; }
    }
    j.bn = best;
    j.nN = (j.N + j.bn - 1) / j.bn;
    j.tiles = j.nM * j.nN;
    return j;
}

__device__ __forceinline__ void cp_async16(unsigned dst, const void * src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(dst), "l"(src) : "memory");
}
// 128 zero bytes: the source of A rows that are zero (an EOU reset's h_prev).
__device__ __align__(128) unsigned char g_zero128[128];

// Arrives on the mbarrier once this thread's earlier cp.async copies have landed
// (the barrier's expected count includes the arrival).
__device__ __forceinline__ void cp_async_arrive(unsigned long long * b) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" :: "r"(smem_u32(b)) : "memory");
}

__device__ __forceinline__ bool err_set(const BulkParams & Q, BulkSmem & S) {
    return *reinterpret_cast<volatile int *>(&S.err) != 0;
}

// Bounded wait on an mbarrier phase; on timeout flags the CTA and the call.
__device__ __forceinline__ bool wait_bar(const BulkParams & Q, BulkSmem & S, unsigned long long * b, unsigned parity) {
    if (mbar_wait(b, parity, Q.P.timeout_ns, &S.err)) return true;
    atomicCAS(&Q.P.ctl[C_ERR], 0, (int) PK_ERR_TIMEOUT);
    return false;
}

// ---- one GEMM phase ------------------------------------------------------------

// Role timing of CTA 0 (one thread per role adds to S.rprof[slot]): 0 A producer
// waiting for a free stage, 1 B producer waiting, 2 MMA waiting for A, 3 MMA waiting
// for B, 4 MMA waiting for a free accumulator, 5 epilogue waiting for an
// accumulator, 6 epilogue work, 7 MMA issue.
struct RoleClock {
    bool on;
    unsigned long long t;
    __device__ __forceinline__ explicit RoleClock(bool enable) : on(enable), t(enable ? gtimer() : 0ull) {}
    __device__ __forceinline__ void add(BulkSmem & S, int slot) {
        if (on) {
            const unsigned long long n = gtimer();
            S.rprof[slot] += n - t;
            t = n;
        }
    }
    __device__ __forceinline__ void skip() {
        if (on) t = gtimer();
    }
};

// A producer (warps 0-3): warp w stages rows 32w .. 32w + 31 of every tile. Its
// lanes first write those rows' sources to a per-warp table in shared memory;
// then each K stage takes 8 rounds of 4 rows x 8 lanes, each lane one 16-byte
// chunk per plane, so that a round reads 4 whole 128-byte row segments
// (coalesced) and writes chunk c of row r at chunk c ^ (r & 7) (128-byte swizzle).
__device__ void gemm_produce_a(const BulkParams & Q, BulkSmem & S, unsigned char * tiles, const Job & J, Pipe & pp) {
    const LoopParams & P = Q.P;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Ring R = ring(J.bn, J.planes);
    const bool lo = J.planes == 2;
    int kk = 0;                                   // K stages of this phase so far
    const int H = P.H, L = P.L, B = P.B;
    const unsigned rb16 = 4u * (unsigned) H;
    // offset of the lo plane in a row: f16 halves (2 bytes a value) or int8 digits
    const unsigned plane = J.kind == G_JOINT ? 2u * (unsigned) P.J : (J.g->i8 ? 1u : 2u) * (unsigned) H;
    for (int t = blockIdx.x; t < J.tiles; t += gridDim.x) {
        {   // this warp's rows: segment 0 for K stages [0, split), segment 1 for the rest
            const int lr = warp * 32 + lane;
            const int row = (t % J.nM) * kBM + lr;
            const unsigned char * src0 = nullptr;
            const unsigned char * src1 = nullptr;
            int r1 = Q.h16_zero_row;
            unsigned char fl = 0;                 // bit 0: row in the batch, bit 1: segment 1 is zero
            if (row < J.M) {
                fl = 1;
                if (J.kind == G_JOINT) {
                    src1 = P.hidc + (size_t) row * P.rbj;
                } else {
                    const int2 e = __ldcg(reinterpret_cast<const int2 *>(P.emit) + row);
                    if (J.kind == G_PRED) {
                        src1 = Q.x16 + ((size_t) (L - 1) * B + row) * rb16;
                    } else {
                        const int hb = (e.y >> 30) & 1;
                        if (e.y < 0) fl |= 2;             // reset: h_prev = 0
                        src1 = Q.h16 + (((size_t) (hb ^ 1) * L + J.l) * B + e.x) * rb16;
                        if (e.y >= 0) r1 = ((hb ^ 1) * L + J.l) * B + e.x;
                        src0 = J.l > 0 ? Q.x16 + ((size_t) (J.l - 1) * B + row) * rb16
                                       : Q.e16 + (size_t) (e.y & 0x3FFFFFFF) * rb16;
                    }
                }
            }
            S.a_s0[lr] = src0;
            S.a_s1[lr] = src1;
            S.a_r1[lr] = r1;
            S.a_fl[lr] = fl;
            __syncwarp();
        }
        for (int kc = 0; kc < J.nK; ++kc, ++kk) {
            const int s = kk % R.n;
            const unsigned u = pp.ua[s]++;
            RoleClock rc(Q.prof != nullptr && blockIdx.x == 0 && threadIdx.x == 0);
            const bool ok = wait_bar(Q, S, &S.empty[s], (u & 1u) ^ 1u);
            rc.add(S, 0);
            if (!__all_sync(0xFFFFFFFFu, ok)) return;
            const bool seg1 = kc >= J.split;
            const unsigned dst = smem_u32(tiles + (unsigned) s * R.stage);
            // compact rows (the joint's hidden rows, the pred-proj input and the lower layer's
            // new h: consecutive list positions) arrive as TMA boxes; h_prev, by utterance,
            // is gathered with cp.async
            if (Q.tma_a && (seg1 ? J.kind != G_LSTM : J.l > 0)) {
                if (threadIdx.x == 0) {
                    const CUtensorMap * map = reinterpret_cast<const CUtensorMap *>(
                        J.kind == G_JOINT ? Q.map_hid : Q.map_x16);
                    const int m0 = (t % J.nM) * kBM;
                    const int y = J.kind == G_JOINT ? m0 : (J.kind == G_PRED ? L - 1 : J.l - 1) * B + m0;
                    const int x = (seg1 ? kc - J.split : kc) * 128;
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                                 :: "r"(smem_u32(&S.full_a[s])), "r"((lo ? 2u : 1u) * kATile) : "memory");
                    tma_load_2d(tiles + (unsigned) s * R.stage, map, x, y, &S.full_a[s]);
                    if (lo) tma_load_2d(tiles + (unsigned) s * R.stage + kATile, map, x + (int) plane, y, &S.full_a[s]);
                } else {
                    mbar_arrive(&S.full_a[s]);
                }
                continue;
            }
            if (Q.tma_a && seg1 && J.kind == G_LSTM) {
                // h_prev rows by utterance: each warp's 32 rows as 8 gather4 loads per plane
                // (lanes 0-7 the hi plane, 8-15 the lo plane); lane 0 posts the warp's bytes
                if (lane == 0)
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                                 :: "r"(smem_u32(&S.full_a[s])), "r"((lo ? 2u : 1u) * 32u * 128u) : "memory");
                __syncwarp();
                if (lane < (lo ? 16 : 8)) {
                    const int r0 = warp * 32 + 4 * (lane & 7);
                    const int pl = lane >> 3;
                    const unsigned d = dst + (unsigned) pl * kATile + (unsigned) r0 * 128u;
                    const int x = (kc - J.split) * 128 + pl * (int) plane;
                    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
                                 " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
                                 :: "r"(d), "l"(reinterpret_cast<const CUtensorMap *>(Q.map_h16)), "r"(x),
                                    "r"(S.a_r1[r0]), "r"(S.a_r1[r0 + 1]), "r"(S.a_r1[r0 + 2]), "r"(S.a_r1[r0 + 3]),
                                    "r"(smem_u32(&S.full_a[s]))
                                 : "memory");
                }
                if (lane != 0) mbar_arrive(&S.full_a[s]);
                continue;
            }
            const unsigned sub = (unsigned) lane & 7u;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int lr = warp * 32 + k * 4 + (lane >> 3);
                const unsigned char fl = S.a_fl[lr];
                if (fl & 1) {
                    // a reset row reads zeros (from a zero block, so that every write of
                    // the stage is a cp.async the arrival below tracks)
                    const bool zero = seg1 && (fl & 2);
                    const unsigned char * shi = zero ? g_zero128
                                              : seg1 ? S.a_s1[lr] + (size_t) (kc - J.split) * 128
                                                     : S.a_s0[lr] + (size_t) kc * 128;
                    const unsigned char * slo = zero ? g_zero128 : shi + plane;
                    const unsigned o = (unsigned) lr * 128u + ((sub ^ ((unsigned) lr & 7u)) << 4);
                    cp_async16(dst + o, shi + sub * 16);
                    if (lo) cp_async16(dst + kATile + o, slo + sub * 16);
                }
            }
            // no wait here: the arrival fires when the copies land (the MMA thread
            // orders them for the tensor cores with a proxy fence after its wait)
            cp_async_arrive(&S.full_a[s]);
        }
        __syncwarp();                             // every lane is done with the table
    }
}

// B producer (warp 4, one lane): the tile's weight rows, hi and lo planes, as
// 64-row TMA boxes (rows past N arrive as zeros).
__device__ void gemm_produce_b(const BulkParams & Q, BulkSmem & S, unsigned char * tiles, const Job & J, Pipe & pp) {
    const CUtensorMap * mhi = reinterpret_cast<const CUtensorMap *>(J.g->map_hi);
    const CUtensorMap * mlo = reinterpret_cast<const CUtensorMap *>(J.g->map_lo);
    const Ring R = ring(J.bn, J.planes);
    int kk = 0;
    for (int t = blockIdx.x; t < J.tiles; t += gridDim.x) {
        const int n0 = (t / J.nM) * J.bn;
        const int rows = min(J.bn, J.N - n0);
        const int nb = (rows + 63) / 64;
        for (int kc = 0; kc < J.nK; ++kc, ++kk) {
            const int s = kk % R.n;
            const unsigned u = pp.ub[s]++;
            RoleClock rc(Q.prof != nullptr && blockIdx.x == 0);
            if (!wait_bar(Q, S, &S.empty[s], (u & 1u) ^ 1u)) return;
            rc.add(S, 1);
            unsigned char * bhi = tiles + (unsigned) s * R.stage + R.b_off;
            unsigned char * blo = bhi + R.b_plane;
            const unsigned planes = (J.g->lo_zero || J.planes == 1) ? 1u : 2u;
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                         :: "r"(smem_u32(&S.full_b[s])), "r"((unsigned) nb * planes * kBBox) : "memory");
            for (int b = 0; b < nb; ++b) {
                tma_load_2d(bhi + b * kBBox, mhi, kc * J.kel, n0 + 64 * b, &S.full_b[s]);
                if (planes == 2u) tma_load_2d(blo + b * kBBox, mlo, kc * J.kel, n0 + 64 * b, &S.full_b[s]);
            }
        }
    }
}

// MMA issuer (warp 5, one lane): per K stage and 16-wide K step, three products
// into the tile's accumulator (columns acc * 256).
__device__ void gemm_mma(const BulkParams & Q, BulkSmem & S, unsigned char * tiles, unsigned tmem, const Job & J,
                         Pipe & pp) {
    const Ring R = ring(J.bn, J.planes);
    const bool three = J.planes == 2 && !J.g->lo_zero;
    int kk = 0;
    for (int t = blockIdx.x; t < J.tiles; t += gridDim.x) {
        const int n0 = (t / J.nM) * J.bn;
        const int rows = min(J.bn, J.N - n0);
        const int nmma = (rows + 15) & ~15;
        const bool i8 = J.g->i8 != 0;
        const unsigned idesc = i8 ? umma_idesc_s8(kBM, nmma) : umma_idesc_f16(kBM, nmma);
        const unsigned a = pp.acc_m & 1u, aph = (pp.acc_m >> 1) & 1u;
        ++pp.acc_m;
        RoleClock rc(Q.prof != nullptr && blockIdx.x == 0);
        if (!wait_bar(Q, S, &S.acc_empty[a], aph ^ 1u)) return;
        rc.add(S, 4);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const unsigned d = tmem + a * (unsigned) kBNmax;
        for (int kc = 0; kc < J.nK; ++kc, ++kk) {
            const int s = kk % R.n;
            const unsigned ph = pp.um[s]++ & 1u;
            rc.skip();
            if (!wait_bar(Q, S, &S.full_a[s], ph)) return;
            rc.add(S, 2);
            if (!wait_bar(Q, S, &S.full_b[s], ph)) return;
            rc.add(S, 3);
            // the A stage was written by cp.async in the generic proxy: make it visible
            // to the tensor cores' (async proxy) reads
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const unsigned base = smem_u32(tiles + (unsigned) s * R.stage);
            const unsigned ahi = base, alo = base + kATile, bhi = base + R.b_off, blo = bhi + R.b_plane;
            if (i8) {
                // int16 digits A = 256 A_hi + A_lo, W = 256 W_hi + W_lo (signed bytes): the
                // 2^16 level A_hi W_hi into columns [0, 128), the 2^8 level A_hi W_lo + A_lo W_hi
                // into [128, 256); the 2^0 level A_lo W_lo is dropped (< 2^-14 of a term's size)
                const unsigned dm = d + (unsigned) (kBNmax / 2);
#pragma unroll
                for (int k32 = 0; k32 < 4; ++k32) {
                    const unsigned ko = (unsigned) k32 * 32u;
                    const unsigned first = (kc | k32) ? 1u : 0u;
                    umma_i8(d, umma_desc_sw128(ahi + ko), umma_desc_sw128(bhi + ko), idesc, first);
                    umma_i8(dm, umma_desc_sw128(ahi + ko), umma_desc_sw128(blo + ko), idesc, first);
                    umma_i8(dm, umma_desc_sw128(alo + ko), umma_desc_sw128(bhi + ko), idesc, 1u);
                }
            } else {
#pragma unroll
                for (int k16 = 0; k16 < kBK / 16; ++k16) {
                    const unsigned ko = (unsigned) k16 * 32u;
                    umma_f16(d, umma_desc_sw128(ahi + ko), umma_desc_sw128(bhi + ko), idesc, (kc | k16) ? 1u : 0u);
                    if (J.planes == 2) umma_f16(d, umma_desc_sw128(alo + ko), umma_desc_sw128(bhi + ko), idesc, 1u);
                    if (three) umma_f16(d, umma_desc_sw128(ahi + ko), umma_desc_sw128(blo + ko), idesc, 1u);
                }
            }
            umma_commit(&S.empty[s]);      // the stage is free once these MMAs have read it
            rc.add(S, 7);
        }
        umma_commit(&S.acc_full[a]);       // the tile's accumulator is complete
    }
}

__device__ __forceinline__ void tmem_ld32(unsigned taddr, float (&v)[32]) {
    unsigned u[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
                   "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]),
                   "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]),
                   "=r"(u[22]), "=r"(u[23]), "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]),
                   "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(u[i]);
}

// f16 hi / lo halves of 8 values, as two 16-byte vectors.
__device__ __forceinline__ void split8(const float (&x)[8], uint4 & hi, uint4 & lo) {
    unsigned h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half a = __float2half_rn(x[2 * i]), b = __float2half_rn(x[2 * i + 1]);
        const __half la = __float2half_rn(x[2 * i] - __half2float(a));
        const __half lb = __float2half_rn(x[2 * i + 1] - __half2float(b));
        __half2 hh = __halves2half2(a, b), ll = __halves2half2(la, lb);
        h[i] = *reinterpret_cast<unsigned *>(&hh);
        l[i] = *reinterpret_cast<unsigned *>(&ll);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Logistic and tanh from the hardware exponential (relative error ~1e-6, against
// a tolerance of 2e-3 on the state; both saturate correctly for large |x|).
__device__ __forceinline__ float sig_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float tanh_fast(float x) { return 1.0f - __fdividef(2.0f, 1.0f + __expf(2.0f * x)); }

// The persistent loop's staged row of 8 new h values at unit j0 (it continues the
// batch): int16 fixed point as two int8 digit planes, or the f16 hi / lo halves.
__device__ __forceinline__ void put_h8(const LoopParams & P, unsigned char * row, int j0, const float (&hn)[8],
                                       const uint4 & hi, const uint4 & lo) {
    if (P.h_int) {
        unsigned dh[2] = {0u, 0u}, dl[2] = {0u, 0u};
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int q16 = max(-32767, min(32767, __float2int_rn(hn[u] * 32768.0f)));
            dh[u >> 2] |= ((unsigned) (q16 >> 8) & 255u) << (8 * (u & 3));
            dl[u >> 2] |= ((unsigned) q16 & 255u) << (8 * (u & 3));
        }
        *reinterpret_cast<uint2 *>(row + j0) = make_uint2(dh[0], dh[1]);
        *reinterpret_cast<uint2 *>(row + P.H + j0) = make_uint2(dl[0], dl[1]);
    } else {
        *reinterpret_cast<uint4 *>(row + 2 * j0) = hi;
        *reinterpret_cast<uint4 *>(row + 2 * P.H + 2 * j0) = lo;
    }
}

// int8 matrices: h (|h| < 1) as int16 fixed point A = round(h * kHScale), split into
// signed digits A = 256 hi + lo (hi = floor((A + 128) / 256), lo in [-128, 127]).
constexpr float kHScale = 32639.0f;                   // |A| <= 32639 keeps hi in [-127, 127]

// 8 new h values at unit j0 into a bulk row of int8 digits: hi at +j0, lo at +H + j0.
__device__ __forceinline__ void put_h8_i8(unsigned char * row, int H, int j0, const float (&hn)[8]) {
    unsigned dh[2] = {0u, 0u}, dl[2] = {0u, 0u};
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int a = max(-32639, min(32639, __float2int_rn(hn[u] * kHScale)));
        const int hi = (a + 128) >> 8;                  // arithmetic shift: floor division
        const int lo = a - 256 * hi;
        dh[u >> 2] |= ((unsigned) hi & 255u) << (8 * (u & 3));
        dl[u >> 2] |= ((unsigned) lo & 255u) << (8 * (u & 3));
    }
    *reinterpret_cast<uint2 *>(row + j0) = make_uint2(dh[0], dh[1]);
    *reinterpret_cast<uint2 *>(row + H + j0) = make_uint2(dl[0], dl[1]);
}

// 8 columns of tensor memory (32x32b shape: this thread's lane), as raw 32-bit words.
__device__ __forceinline__ void tmem_ld8(unsigned taddr, unsigned (&u)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7])
                 : "r"(taddr));
}

// The two int8 accumulators of 32 columns: value = (2^16 acc_hh + 2^8 acc_m) * rscale / kHScale
// (8 columns of each level at a time, to keep few registers live).
__device__ __forceinline__ void tmem_ld32_i8(unsigned tacc, int c0, const float * rscale, float (&v)[32]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        unsigned hh[8], mm[8];
        tmem_ld8(tacc + (unsigned) (c0 + 8 * k), hh);
        tmem_ld8(tacc + (unsigned) (kBNmax / 2 + c0 + 8 * k), mm);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const float4 r0 = __ldg(reinterpret_cast<const float4 *>(rscale) + 2 * k);
        const float4 r1 = __ldg(reinterpret_cast<const float4 *>(rscale) + 2 * k + 1);
        const float rs[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float t = (float) (int) hh[q] * 65536.0f + (float) (int) mm[q] * 256.0f;
            v[8 * k + q] = t * (rs[q] * (1.0f / kHScale));
        }
    }
}

// Epilogue of an LSTM layer: the tile's columns are gates (i, f, g, o) of units
// [n0 / 4, (n0 + rows) / 4); row = emit-list index. Every 8 units take one
// tensor-memory load of their 32 gate sums; their old cell state was requested
// one group earlier.
__device__ __forceinline__ void epi_lstm(const BulkParams & Q, const Job & J, unsigned tacc, int row, int n0, int rows) {
    const LoopParams & P = Q.P;
    const int H = P.H, L = P.L, B = P.B, l = J.l;
    const bool valid = row < J.M;
    const bool i8 = J.g->i8 != 0;
    int utt = 0, hb = 0, reset = 1, tok = 0;
    if (valid) {
        const int2 e = __ldcg(reinterpret_cast<const int2 *>(P.emit) + row);
        utt = e.x;
        hb = (e.y >> 30) & 1;
        reset = e.y < 0 ? 1 : 0;
        tok = e.y & 0x3FFFFFFF;
    }
    const unsigned rb16 = 4u * (unsigned) H;
    const float * crow = P.c + ((size_t) l * B + utt) * H;
    float * cw = P.c + ((size_t) l * B + utt) * H;
    float * hw = P.h + (((size_t) hb * L + l) * B + utt) * H;
    unsigned char * st = Q.h16 + (((size_t) hb * L + l) * B + utt) * rb16;
    unsigned char * xn = Q.x16 + ((size_t) l * B + row) * rb16;
    // int8 layer 0: its input projection and both biases come from the token's table row
    const float * bias = (i8 && l == 0) ? Q.g0b + (size_t) tok * 4 * H : Q.lbias + (size_t) l * 4 * H;
    // next group's old cell state is requested before this group's tensor-memory load
    float4 cn0 = make_float4(0.f, 0.f, 0.f, 0.f), cn1 = cn0;
    if (valid && !reset && rows > 0) {
        cn0 = __ldcg(reinterpret_cast<const float4 *>(crow + (n0 >> 2)));
        cn1 = __ldcg(reinterpret_cast<const float4 *>(crow + (n0 >> 2)) + 1);
    }
    for (int c0 = 0; c0 < rows; c0 += 32) {
        const float4 co0 = cn0, co1 = cn1;
        if (valid && !reset && c0 + 32 < rows) {
            cn0 = __ldcg(reinterpret_cast<const float4 *>(crow + ((n0 + c0 + 32) >> 2)));
            cn1 = __ldcg(reinterpret_cast<const float4 *>(crow + ((n0 + c0 + 32) >> 2)) + 1);
        }
        float v[32];
        if (i8) tmem_ld32_i8(tacc, c0, J.g->rscale + n0 + c0, v);   // warp-wide: every lane takes part
        else tmem_ld32(tacc + (unsigned) c0, v);
        if (!valid) continue;
        const int j0 = (n0 + c0) >> 2;                      // first of the 8 units in these columns
        const float4 * b4 = reinterpret_cast<const float4 *>(bias + 4 * j0);
        const float cold[8] = {co0.x, co0.y, co0.z, co0.w, co1.x, co1.y, co1.z, co1.w};
        float hn[8], cn[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const float4 bb = __ldg(b4 + u);
            const float i_g = sig_fast(bb.x + v[4 * u + 0]);
            const float f_g = sig_fast(bb.y + v[4 * u + 1]);
            const float g_g = tanh_fast(bb.z + v[4 * u + 2]);
            const float o_g = sig_fast(bb.w + v[4 * u + 3]);
            cn[u] = f_g * cold[u] + i_g * g_g;
            hn[u] = o_g * tanh_fast(cn[u]);
        }
        reinterpret_cast<float4 *>(cw + j0)[0] = make_float4(cn[0], cn[1], cn[2], cn[3]);
        reinterpret_cast<float4 *>(cw + j0)[1] = make_float4(cn[4], cn[5], cn[6], cn[7]);
        if (P.trace_steps > 0) {   // f32 h: only the trace's state dump reads it
            reinterpret_cast<float4 *>(hw + j0)[0] = make_float4(hn[0], hn[1], hn[2], hn[3]);
            reinterpret_cast<float4 *>(hw + j0)[1] = make_float4(hn[4], hn[5], hn[6], hn[7]);
        }
        if (i8) {
            put_h8_i8(st, H, j0, hn);
            put_h8_i8(xn, H, j0, hn);
        } else {
            uint4 hi, lo;
            split8(hn, hi, lo);
            *reinterpret_cast<uint4 *>(st + 2 * j0) = hi;
            *reinterpret_cast<uint4 *>(st + 2 * H + 2 * j0) = lo;
            *reinterpret_cast<uint4 *>(xn + 2 * j0) = hi;
            *reinterpret_cast<uint4 *>(xn + 2 * H + 2 * j0) = lo;
        }
    }
}

__device__ __forceinline__ void epi_pred(const BulkParams & Q, const Job & J, unsigned tacc, int row, int n0, int rows) {
    const LoopParams & P = Q.P;
    const bool valid = row < J.M;
    const int utt = valid ? __ldcg(&P.emit[2 * row]) : 0;
    for (int c0 = 0; c0 < rows; c0 += 32) {
        float v[32];
        if (J.g->i8) tmem_ld32_i8(tacc, c0, J.g->rscale + n0 + c0, v);
        else tmem_ld32(tacc + (unsigned) c0, v);
        if (!valid) continue;
        float * o = P.predp + (size_t) utt * P.J + n0 + c0;
        const float * b = P.pred_b + n0 + c0;
#pragma unroll
        for (int q = 0; q < 32; q += 4) {
            if (n0 + c0 + q < P.J)
                *reinterpret_cast<float4 *>(o + q) = make_float4(v[q] + __ldg(b + q), v[q + 1] + __ldg(b + q + 1),
                                                                 v[q + 2] + __ldg(b + q + 2), v[q + 3] + __ldg(b + q + 3));
        }
    }
}

// Joint epilogue: logits = bias + acc over the tile's rows of joint.out; the first
// index of the largest token logit and of the largest duration logit of the tile
// (strict >, in index order, as argmax_f32 scans) become one 64-bit key each,
// max-reduced over the tiles of the row.
__device__ __forceinline__ void epi_joint(const BulkParams & Q, const Job & J, unsigned tacc, int row, int n0,
                                          int rows, unsigned long long * keys) {
    const LoopParams & P = Q.P;
    const bool valid = row < J.M;
    int utt = 0, step = 0;
    if (valid) {
        utt = __ldcg(P.live + (size_t) J.sel * P.B + row);
        if (P.trace_steps > 0) step = __ldcg(&P.ust[utt * kUst + U_STEPS]);
    }
    const bool tr = valid && P.trace_steps > 0 && step < P.trace_steps;
    float bt = 0.0f, bd = 0.0f;
    int it = -1, id = -1;
    for (int c0 = 0; c0 < rows; c0 += 32) {
        float v[32];
        tmem_ld32(tacc + (unsigned) c0, v);
        if (!valid) continue;
        const int r0 = n0 + c0;
        const bool full = r0 + 32 <= P.Vo;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
            if (full) {
                bb = __ldg(reinterpret_cast<const float4 *>(P.out_b + r0) + k);
            } else {
                const int r = r0 + 4 * k;
                bb.x = r < P.Vo ? __ldg(P.out_b + r) : 0.f;
                bb.y = r + 1 < P.Vo ? __ldg(P.out_b + r + 1) : 0.f;
                bb.z = r + 2 < P.Vo ? __ldg(P.out_b + r + 2) : 0.f;
                bb.w = r + 3 < P.Vo ? __ldg(P.out_b + r + 3) : 0.f;
            }
            const float lg[4] = {bb.x + v[4 * k], bb.y + v[4 * k + 1], bb.z + v[4 * k + 2], bb.w + v[4 * k + 3]};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int r = r0 + 4 * k + q;
                if (r < P.Vo) {
                    if (tr) P.tr_logits[((size_t) utt * P.trace_steps + step) * P.Vo + r] = lg[q];
                    if (r < P.V1) {
                        if (it < 0 || lg[q] > bt) { bt = lg[q]; it = r; }
                    } else {
                        if (id < 0 || lg[q] > bd) { bd = lg[q]; id = r - P.V1; }
                    }
                }
            }
        }
    }
    if (valid) {
        if (it >= 0) atomicMax(&keys[2 * utt + 0], make_key(bt, it));
        if (id >= 0) atomicMax(&keys[2 * utt + 1], make_key(bd, id));
    }
}

// Screened joint epilogue: the tile's approximate token logits (bias + A_hi W_hi) are
// reduced to their four largest values and the indices of the first three, written to
// the row's summary slot for this N tile; duration columns are left to the decision,
// which computes them in f32. A NaN among the tile's logits sets the slot's flag so
// that the decision falls back to the full index-order scan.
__device__ __forceinline__ void epi_joint_screen(const BulkParams & Q, const Job & J, unsigned tacc, int row, int n0,
                                                 int rows, int nt) {
    const LoopParams & P = Q.P;
    const bool valid = row < J.M;
    const int tok_end = min(rows, P.V1 - n0);          // token columns: [n0, n0 + tok_end)
    float m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY, m4 = -INFINITY;
    unsigned j1 = 0xFFFFFFFFu, j2 = 0xFFFFFFFFu, j3 = 0xFFFFFFFFu;
    bool nan = false;
    for (int c0 = 0; c0 < rows; c0 += 32) {
        float v[32];
        tmem_ld32(tacc + (unsigned) c0, v);                 // warp-wide: every lane takes part
        if (c0 >= tok_end) continue;                        // the same for the whole warp
        const int r0 = n0 + c0;
        const int cnt = min(32, tok_end - c0);
        float lg[32];
        if (cnt == 32) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float4 bb = __ldg(reinterpret_cast<const float4 *>(P.out_b + r0) + k);
                lg[4 * k + 0] = bb.x + v[4 * k + 0];
                lg[4 * k + 1] = bb.y + v[4 * k + 1];
                lg[4 * k + 2] = bb.z + v[4 * k + 2];
                lg[4 * k + 3] = bb.w + v[4 * k + 3];
            }
        } else {
#pragma unroll
            for (int q = 0; q < 32; ++q) lg[q] = q < cnt ? __ldg(P.out_b + r0 + q) + v[q] : -INFINITY;
        }
        // branch-free insertion into m1 >= m2 >= m3 >= m4 (strict > keeps the earlier
        // index first among equal values)
#pragma unroll
        for (int q = 0; q < 32; ++q) {
            const float x = lg[q];
            const unsigned jq = (unsigned) (r0 + q);
            nan |= x != x;
            const bool g1 = x > m1, g2 = x > m2, g3 = x > m3, g4 = x > m4;
            m4 = g3 ? m3 : (g4 ? x : m4);
            m3 = g2 ? m2 : (g3 ? x : m3);
            j3 = g2 ? j2 : (g3 ? jq : j3);
            m2 = g1 ? m1 : (g2 ? x : m2);
            j2 = g1 ? j1 : (g2 ? jq : j2);
            m1 = g1 ? x : m1;
            j1 = g1 ? jq : j1;
        }
    }
    if (valid) {
        uint4 * d = Q.jsum + ((size_t) row * Q.jsum_stride + nt) * 2;
        d[0] = make_uint4(__float_as_uint(m1), __float_as_uint(m2), __float_as_uint(m3), __float_as_uint(m4));
        d[1] = make_uint4(j1, j2, j3, nan ? 1u : 0u);
    }
}

// Epilogue warps 8-11: warp % 4 selects the TMEM lane quarter = rows 32 (warp % 4) .. + 31.
__device__ void gemm_epilogue(const BulkParams & Q, BulkSmem & S, unsigned tmem, const Job & J, Pipe & pp,
                              unsigned long long * keys) {
    const int quarter = (threadIdx.x >> 5) & 3, lane = threadIdx.x & 31;
    for (int t = blockIdx.x; t < J.tiles; t += gridDim.x) {
        const int row = (t % J.nM) * kBM + quarter * 32 + lane;
        const int n0 = (t / J.nM) * J.bn;
        const int rows = min(J.bn, J.N - n0);
        const unsigned a = pp.acc_e & 1u, aph = (pp.acc_e >> 1) & 1u;
        ++pp.acc_e;
        RoleClock rc(Q.prof != nullptr && blockIdx.x == 0 && threadIdx.x == 256);
        if (!wait_bar(Q, S, &S.acc_full[a], aph)) return;
        rc.add(S, 5);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const unsigned tacc = tmem + ((unsigned) (quarter * 32) << 16) + a * (unsigned) kBNmax;
        if (J.kind == G_LSTM) epi_lstm(Q, J, tacc, row, n0, rows);
        else if (J.kind == G_PRED) epi_pred(Q, J, tacc, row, n0, rows);
        else if (J.planes == 1) epi_joint_screen(Q, J, tacc, row, n0, rows, t / J.nM);
        else epi_joint(Q, J, tacc, row, n0, rows, keys);
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        rc.add(S, 6);
        mbar_arrive(&S.acc_empty[a]);
    }
}

// Every thread of the CTA: its role's share of the phase. False if a wait gave up.
__device__ bool gemm_phase(const BulkParams & Q, BulkSmem & S, unsigned char * tiles, unsigned tmem, const Job & J,
                           Pipe & pp, unsigned long long * keys) {
    const int warp = threadIdx.x >> 5;
    if (J.tiles > 0) {
        if (warp < 4) gemm_produce_a(Q, S, tiles, J, pp);
        else if (warp == 4) {
            if ((threadIdx.x & 31) == 0) gemm_produce_b(Q, S, tiles, J, pp);
            __syncwarp();
        } else if (warp == 5) {
            if ((threadIdx.x & 31) == 0) gemm_mma(Q, S, tiles, tmem, J, pp);
            __syncwarp();
        }
        else if (warp >= 8) gemm_epilogue(Q, S, tmem, J, pp, keys);
    }
    return __syncthreads_or(err_set(Q, S) ? 1 : 0) == 0;
}

// ---- grid barrier and block scan -------------------------------------------------

// k-th barrier of this launch on the counter P.bar[6] (zeroed by the host).
__device__ bool bulk_barrier(const BulkParams & Q, BulkSmem & S, unsigned & k) {
    const LoopParams & P = Q.P;
    __syncthreads();
    const unsigned target = (k + 1u) * gridDim.x;
    ++k;
    if (threadIdx.x == 0) {
        red_add_release(&P.bar[6], 1u);
        int ok = 1;
        const unsigned long long t0 = gtimer();
        for (unsigned it = 1;; ++it) {
            if ((int) (ld_acquire(&P.bar[6]) - target) >= 0) break;
            if ((it & 63u) == 0u) {
                if (__ldcg(&P.ctl[C_ERR]) != 0) { ok = 0; break; }
                if ((long long) (gtimer() - t0) > P.timeout_ns) {
                    atomicCAS(&P.ctl[C_ERR], 0, (int) PK_ERR_TIMEOUT);
                    ok = 0;
                    break;
                }
            }
        }
        S.flag[0] = ok;
    }
    __syncthreads();
    return S.flag[0] != 0;
}

__device__ int bulk_scan(BulkSmem & S, int v, int & total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) S.scan[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const int w = lane < kBWarps ? S.scan[lane] : 0;
        int y = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int z = __shfl_up_sync(0xFFFFFFFFu, y, o);
            if (lane >= o) y += z;
        }
        if (lane < kBWarps) S.scan[lane] = y - w;
        if (lane == kBWarps - 1) S.scan[kBWarps] = y;
    }
    __syncthreads();
    total = S.scan[kBWarps];
    const int r = x - v + S.scan[warp];
    __syncthreads();
    return r;
}

// ---- element-wise phase: joint hidden layer (and the trace's state dump) ------------

__device__ void hidden_phase(const BulkParams & Q, int sel, int n_live, int n_prev) {
    const LoopParams & P = Q.P;
    const int J = P.J, B = P.B;
    const int q4 = J / 4;
    const long long total = (long long) n_live * q4;
    const long long stride = (long long) gridDim.x * blockDim.x;
    const int * live = P.live + (size_t) sel * B;
    const long long * lfr = reinterpret_cast<const long long *>(P.live_frame) + (size_t) sel * B;
    for (long long idx = (long long) blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
        const int i = (int) (idx / q4), q = (int) (idx - (long long) i * q4);
        const int utt = __ldcg(live + i);
        const long long fr = __ldcg(lfr + i);
        const float4 e = __ldcg(reinterpret_cast<const float4 *>(P.encp + (size_t) fr * J) + q);
        const float4 p = __ldcg(reinterpret_cast<const float4 *>(P.predp + (size_t) utt * J) + q);
        // relu as the persistent loop writes it: (0 < v) ? v : 0
        const float vv[4] = {e.x + p.x, e.y + p.y, e.z + p.z, e.w + p.w};
        float x[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) x[k] = (0.0f < vv[k]) ? vv[k] : 0.0f;
        unsigned char * rowp = P.hidc + (size_t) i * P.rbj;
        __half hh[4], hl[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            hh[k] = __float2half_rn(x[k]);
            hl[k] = __float2half_rn(x[k] - __half2float(hh[k]));
        }
        __half2 h01 = __halves2half2(hh[0], hh[1]), h23 = __halves2half2(hh[2], hh[3]);
        __half2 l01 = __halves2half2(hl[0], hl[1]), l23 = __halves2half2(hl[2], hl[3]);
        *reinterpret_cast<uint2 *>(rowp + 8 * q) =
            make_uint2(*reinterpret_cast<unsigned *>(&h01), *reinterpret_cast<unsigned *>(&h23));
        *reinterpret_cast<uint2 *>(rowp + 2 * J + 8 * q) =
            make_uint2(*reinterpret_cast<unsigned *>(&l01), *reinterpret_cast<unsigned *>(&l23));
        if (screened(Q, n_live)) {
            // ||hid||^2 of the row as the decision's f32 recomputation sees it (hi + lo).
            // J / 4 is a multiple of 32 (bulk_screen_supported) and a warp's 32 indices are
            // consecutive from a multiple of 32, so the whole warp is in row i.
            float ss = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float av = __half2float(hh[k]) + __half2float(hl[k]);
                ss = fmaf(av, av, ss);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
            if ((threadIdx.x & 31) == 0) atomicAdd(Q.norm2 + i, ss);
        }
    }
    // teacher-forced trace: state after each step decided by the previous iteration
    if (P.trace_steps > 0 && n_prev > 0) {
        const int H = P.H, L = P.L, LH = L * H;
        const int * prev = P.live + (size_t) (sel ^ 1) * B;
        const long long tot2 = (long long) n_prev * LH;
        for (long long idx = (long long) blockIdx.x * blockDim.x + threadIdx.x; idx < tot2; idx += stride) {
            const int i = (int) (idx / LH), k = (int) (idx - (long long) i * LH);
            const int utt = __ldcg(prev + i);
            const int step = __ldcg(&P.ust[utt * kUst + U_STEPS]) - 1;
            if (step < 0 || step >= P.trace_steps) continue;
            const int hb = __ldcg(&P.ust[utt * kUst + U_HBUF]);
            const int l = k / H, j = k - (k / H) * H;
            const size_t dst = ((size_t) utt * P.trace_steps + step) * LH + k;
            if (P.tr_h) P.tr_h[dst] = __ldcg(P.h + (((size_t) hb * L + l) * B + utt) * H + j);
            if (P.tr_c) P.tr_c[dst] = __ldcg(P.c + ((size_t) l * B + utt) * H + j);
        }
    }
}

// ---- screened joint: the exact argmax ---------------------------------------------

constexpr int kScreenMaxJ = 1024;          // hidden rows held in registers: J / 32 <= 32 per lane

// f32 logits of kCand joint.out rows (rows[c]; every entry a valid row) for the hidden
// row the warp holds (lane l has a[m] = hid[64 m + 2 l .. + 1]). The weights are read
// as their exact f16 halves (hi + lo, the arrays the joint GEMM streams); every lane
// returns the same values (fixed summation order). N2 = J / 64 is a compile-time
// trip count so that every load can be issued before the first product.
constexpr int kCand = 8;
template <int N2>
__device__ __forceinline__ void exact_logits_n(const BulkParams & Q, const float2 (&a)[kScreenMaxJ / 64],
                                               const int (&rows)[kCand], float (&out)[kCand]) {
    const LoopParams & P = Q.P;
    const int lane = threadIdx.x & 31;
    const __half2 * whi = static_cast<const __half2 *>(Q.gj.hi);
    const __half2 * wlo = static_cast<const __half2 *>(Q.gj.lo);
    const int rs = P.J / 2;                            // half2 per weight row
    float s[kCand];
#pragma unroll
    for (int c = 0; c < kCand; ++c) s[c] = 0.0f;
#pragma unroll
    for (int m = 0; m < N2; ++m) {
#pragma unroll
        for (int c = 0; c < kCand; ++c) {
            const size_t o = (size_t) rows[c] * rs + lane + 32 * m;
            const float2 h = __half22float2(__ldg(whi + o)), l = __half22float2(__ldg(wlo + o));
            s[c] = fmaf(h.y + l.y, a[m].y, fmaf(h.x + l.x, a[m].x, s[c]));
        }
    }
#pragma unroll
    for (int c = 0; c < kCand; ++c) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s[c] += __shfl_xor_sync(0xFFFFFFFFu, s[c], o);
        out[c] = __ldg(P.out_b + rows[c]) + s[c];
    }
}

// rows[0 .. n) with 1 <= n <= kCand; entries past n repeat the last row.
__device__ __forceinline__ void exact_logits(const BulkParams & Q, const float2 (&a)[kScreenMaxJ / 64],
                                             int (&rows)[kCand], int n, float (&out)[kCand]) {
#pragma unroll
    for (int c = 1; c < kCand; ++c)
        if (c >= n) rows[c] = rows[c - 1];
    switch (Q.P.J / 64) {
        case 2: exact_logits_n<2>(Q, a, rows, out); break;
        case 4: exact_logits_n<4>(Q, a, rows, out); break;
        case 6: exact_logits_n<6>(Q, a, rows, out); break;
        case 8: exact_logits_n<8>(Q, a, rows, out); break;
        case 10: exact_logits_n<10>(Q, a, rows, out); break;
        case 12: exact_logits_n<12>(Q, a, rows, out); break;
        case 14: exact_logits_n<14>(Q, a, rows, out); break;
        default: exact_logits_n<16>(Q, a, rows, out); break;
    }
}

// One warp: the token and duration decisions of live row g from the screened joint.
//
// Bound: with w~ = f16(w), a~ = f16(a) (the hi halves the GEMM used) and a = hi + lo
// (the row the f32 recomputation uses), |w a - w~ a~| <= 2^-10 (1 + 2^-11) |w||a| per
// term; the tensor core's f32 accumulation and the recomputation's f32 sums add at most
// (K + 37) 2^-23 sum |w||a| (< 1.3e-4 sum |w||a| for K <= 1024, counting one rounding
// per addition), so the total stays below 2^-9 sum |w||a|; and sum |w||a| <=
// max_j ||w_j|| ||a|| (Cauchy-Schwarz). So every token's approximate logit is within
// E = 2^-9 ||w||max ||a|| (plus a slack for the bias additions) of its recomputed value,
// and the recomputed argmax j* satisfies approx(j*) >= M - 2E, M the largest
// approximate logit. The candidates -- every token with approx >= M - 2E, through each
// N tile's top three, or the whole tile when its fourth value also qualifies, and the
// token rows past the last whole 64-row block, which are not screened -- are
// recomputed in f32 and the largest wins, ties to the smallest index (argmax_f32's
// first-index rule, src/parakeet_tdt.cpp:25-32). A NaN or infinity anywhere sends the
// row to the full index-order scan. The duration logits (TDT) are recomputed with the
// token candidates, and argmax_f32 runs over them.
//
// Memory round trips: (1) the hidden row, the row norm and every tile's top value;
// (2) the full summaries of the tiles that reach the threshold (usually one or two);
// (3) the candidate and duration rows.
__device__ void screen_row(const BulkParams & Q, const Job & JJ, int g, int & tok, int & dur) {
    const LoopParams & P = Q.P;
    const int lane = threadIdx.x & 31;
    const int npair = P.J / 64;                        // half2 pairs per lane
    const __half2 * hi = reinterpret_cast<const __half2 *>(P.hidc + (size_t) g * P.rbj);
    const __half2 * lo = hi + P.J / 2;
    const uint4 * sm = Q.jsum + (size_t) g * Q.jsum_stride * 2;
    float2 a[kScreenMaxJ / 64];
#pragma unroll
    for (int m = 0; m < kScreenMaxJ / 64; ++m) {
        a[m] = make_float2(0.0f, 0.0f);
        if (m < npair) {
            const float2 h = __half22float2(__ldcg(hi + lane + 32 * m)), l = __half22float2(__ldcg(lo + lane + 32 * m));
            a[m] = make_float2(h.x + l.x, h.y + l.y);
        }
    }
    const float n2 = __ldcg(Q.norm2 + g);
    constexpr int kTl = 8;                             // tiles per lane: nN <= 256
    float t1[kTl];
#pragma unroll
    for (int k = 0; k < kTl; ++k) {
        const int t = lane + 32 * k;
        t1[k] = t < JJ.nN ? __ldcg(reinterpret_cast<const float *>(sm + 2 * t)) : -INFINITY;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < kTl; ++k) mx = fmaxf(mx, t1[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    const float E = 0x1p-9f * 1.01f * __ldg(Q.wnorm) * sqrtf(n2) + 1e-5f * (1.0f + fabsf(mx));
    bool wild = !isfinite(mx) || !isfinite(E) || JJ.nN > 32 * kTl;
    const float thr = mx - 2.0f * E;
    // (2) tiles whose top value reaches the threshold: their summaries and NaN flags
    int rows[kCand];
    float v[kCand];
#pragma unroll
    for (int c = 0; c < kCand; ++c) rows[c] = 0;
    int n = 0;
    float best = 0.0f, bd = 0.0f;
    int bj = -1;
    dur = 0;
    // fold the queued rows into (best, bj): largest value, then smallest index; queued
    // duration rows (index >= V1) into (bd, dur) by argmax_f32 (first index of the largest)
    auto flush = [&]() {
        exact_logits(Q, a, rows, n, v);
#pragma unroll
        for (int c = 0; c < kCand; ++c) {
            if (c < n) {
                const int r = rows[c];
                if (r >= P.V1) {
                    const int d = r - P.V1;
                    if (d == 0 || v[c] > bd) { bd = v[c]; dur = d; }
                } else if (bj < 0 || v[c] > best || (v[c] == best && r < bj)) {
                    best = v[c];
                    bj = r;
                }
            }
        }
        n = 0;
    };
    auto push = [&](int j) {
#pragma unroll
        for (int c = 0; c < kCand; ++c)
            if (c == n) rows[c] = j;
        if (++n == kCand) flush();
    };
    if (!wild) {
        // one pass over the lanes' tiles, in tile order (durations are queued first, in
        // index order, so their argmax sees them in order even across flushes; then the
        // unscreened token rows [n_scr, V1))
        if (P.is_tdt)
            for (int d = 0; d < P.Nd; ++d) push(P.V1 + d);
        for (int j = Q.n_scr; j < P.V1; ++j) push(j);
#pragma unroll
        for (int k = 0; k < kTl; ++k) {
            unsigned hit = __ballot_sync(0xFFFFFFFFu, t1[k] >= thr);
            uint4 e0 = make_uint4(0u, 0u, 0u, 0u), e1 = e0;
            if (t1[k] >= thr) {
                e0 = __ldcg(sm + 2 * (lane + 32 * k));
                e1 = __ldcg(sm + 2 * (lane + 32 * k) + 1);
            }
            const bool flag = t1[k] >= thr && e1.w != 0u;
            if (__any_sync(0xFFFFFFFFu, flag)) { wild = true; break; }
            while (hit) {
                const int src = __ffs(hit) - 1;
                hit &= hit - 1;
                const float m2 = __uint_as_float(__shfl_sync(0xFFFFFFFFu, e0.y, src));
                const float m3 = __uint_as_float(__shfl_sync(0xFFFFFFFFu, e0.z, src));
                const float m4 = __uint_as_float(__shfl_sync(0xFFFFFFFFu, e0.w, src));
                const int j1 = (int) __shfl_sync(0xFFFFFFFFu, e1.x, src);
                const int j2 = (int) __shfl_sync(0xFFFFFFFFu, e1.y, src);
                const int j3 = (int) __shfl_sync(0xFFFFFFFFu, e1.z, src);
                if (m4 >= thr) {                       // more than three candidates: the whole tile
                    const int r0 = (32 * k + src) * JJ.bn, r1 = min(r0 + JJ.bn, P.V1);
                    for (int j = r0; j < r1; ++j) push(j);
                } else {
                    push(j1);
                    if (m2 >= thr) push(j2);
                    if (m3 >= thr) push(j3);
                }
            }
        }
    }
    if (!wild) {
        if (n > 0) flush();
        tok = bj;
        return;
    }
    // argmax_f32 over every token, in index order (strict >: only index 0 can win as NaN),
    // then over the durations
    n = 0;
    bj = -1;
    for (int j0 = 0; j0 < P.V1; j0 += kCand) {
        const int cnt = min(kCand, P.V1 - j0);
#pragma unroll
        for (int c = 0; c < kCand; ++c) rows[c] = j0 + min(c, cnt - 1);
        exact_logits(Q, a, rows, cnt, v);
#pragma unroll
        for (int c = 0; c < kCand; ++c)
            if (c < cnt && (j0 + c == 0 || v[c] > best)) { best = v[c]; bj = j0 + c; }
    }
    tok = bj;
    dur = 0;
    if (P.is_tdt) {
        for (int d0 = 0; d0 < P.Nd; d0 += kCand) {
            const int cnt = min(kCand, P.Nd - d0);
#pragma unroll
            for (int c = 0; c < kCand; ++c) rows[c] = P.V1 + d0 + min(c, cnt - 1);
            exact_logits(Q, a, rows, cnt, v);
#pragma unroll
            for (int c = 0; c < kCand; ++c)
                if (c < cnt && (d0 + c == 0 || v[c] > bd)) { bd = v[c]; dur = d0 + c; }
        }
    }
}

// ---- hand-over to the persistent loop ------------------------------------------------

// The persistent loop keeps h in its own staged layout (pk_loop.cu): write both h
// buffers of every layer of every utterance still live or about to take its LSTM
// step into it, from the f16 halves kept here (h = hi + lo, the value this loop
// computed). Only the last buffer written is ever read; the other is written too
// so that nothing needs to know which one that is.
__device__ void handoff_phase(const BulkParams & Q, int sel, int n_live, int n_emit) {
    const LoopParams & P = Q.P;
    const int H = P.H, L = P.L, B = P.B;
    const int groups = H / 8;
    // the live list, then the emit list (its last LSTM step runs on the persistent loop)
    const long long total = (long long) (n_live + n_emit) * 2 * L * groups;
    const long long stride = (long long) gridDim.x * blockDim.x;
    const unsigned rb16 = 4u * (unsigned) H;
    for (long long idx = (long long) blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
        const int g = (int) (idx % groups);
        const long long r = idx / groups;                 // (live entry, buffer, layer)
        const int l = (int) (r % L), hb = (int) ((r / L) % 2), i = (int) (r / (2 * L));
        const int utt = i < n_live ? __ldcg(P.live + (size_t) sel * B + i) : __ldcg(P.emit + 2 * (i - n_live));
        const unsigned char * src = Q.h16 + (((size_t) hb * L + l) * B + utt) * rb16;
        float hn[8];
        uint4 hi, lo;
        if (Q.gl[0].i8) {                                // int16 digits: h = (256 hi + lo) / kHScale
            const uint2 dh = __ldcg(reinterpret_cast<const uint2 *>(src + 8 * g));
            const uint2 dl = __ldcg(reinterpret_cast<const uint2 *>(src + H + 8 * g));
            const signed char * ch = reinterpret_cast<const signed char *>(&dh);
            const signed char * cl = reinterpret_cast<const signed char *>(&dl);
#pragma unroll
            for (int u = 0; u < 8; ++u) hn[u] = (float) (256 * (int) ch[u] + (int) cl[u]) * (1.0f / kHScale);
            split8(hn, hi, lo);
        } else {
            hi = __ldcg(reinterpret_cast<const uint4 *>(src + 16 * g));
            lo = __ldcg(reinterpret_cast<const uint4 *>(src + 2 * H + 16 * g));
            const __half * hh = reinterpret_cast<const __half *>(&hi);
            const __half * hl = reinterpret_cast<const __half *>(&lo);
#pragma unroll
            for (int u = 0; u < 8; ++u) hn[u] = __half2float(hh[u]) + __half2float(hl[u]);
        }
        put_h8(P, P.hst + ((((size_t) hb * L + l) * B + utt) * P.rbh), 8 * g, hn, hi, lo);
    }
}

// ---- the kernel -------------------------------------------------------------------

__global__ void __launch_bounds__(kBThreads, 1) bulk_loop_kernel(const __grid_constant__ BulkParams Q) {
    const LoopParams & P = Q.P;
    extern __shared__ __align__(1024) unsigned char bk_raw[];
    unsigned char * tiles = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(bk_raw) + 1023) & ~(uintptr_t) 1023);
    BulkSmem & S = *reinterpret_cast<BulkSmem *>(tiles + kRing);
    const int warp = threadIdx.x >> 5;
    const int G = (int) gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxStages; ++s) {
            mbar_init(&S.full_a[s], 128);
            mbar_init(&S.full_b[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&S.acc_full[a], 1);
            mbar_init(&S.acc_empty[a], 128);
        }
        S.err = 0;
        for (int i = 0; i < 8; ++i) S.rprof[i] = 0ull;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(&S.tmem_base)), "r"(kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tmem = S.tmem_base;
    if (blockIdx.x == 0 && threadIdx.x == 0) *P.t_start = gtimer();

    Pipe pp;
    unsigned nbar = 0;
    // CTA 0's thread 0 times every phase: [2k] its own share, [2k + 1] the grid barrier
    // after it (k: 0 LSTM layers, 1 pred-proj, 2 joint hidden, 3 joint, 4 decision,
    // 5 list compaction)
    const bool prof = blockIdx.x == 0 && threadIdx.x == 0 && Q.prof != nullptr;
    unsigned long long pacc[12] = {0ull, 0ull, 0ull, 0ull, 0ull, 0ull, 0ull, 0ull, 0ull, 0ull, 0ull, 0ull};
    unsigned long long plast = prof ? gtimer() : 0ull;
    auto mark = [&](int slot) {
        if (prof) {
            const unsigned long long now = gtimer();
            pacc[slot] += now - plast;
            plast = now;
        }
    };
    int sel = __ldcg(&P.ctl[C_SEL]);
    int n_emit = __ldcg(&P.ctl[C_NEMIT]);
    int n_live = __ldcg(&P.ctl[C_NLIVE0 + sel]);
    int n_prev = 0, iter = 0, emit_iters = 0;
    long long sum_live = 0, sum_emit = 0;    // this loop's joint evaluations and LSTM steps
    long long sum_scr = 0;                   // of them, screened joint evaluations
    unsigned long long * keys = P.keys;                 // one key buffer: cleared by the decision that reads it
    bool ok = __ldcg(&P.ctl[C_ERR]) == 0;
    while (ok && n_live >= Q.min_live && n_live > 0) {
        if (iter > P.max_iters) {
            if (blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(&P.ctl[C_ERR], 0, (int) PK_ERR_DEVICE);
            break;
        }
        if (n_emit > 0) {
            ++emit_iters;
            for (int l = 0; l < P.L && ok; ++l) {
                ok = gemm_phase(Q, S, tiles, tmem, make_job(Q, G_LSTM, l, n_emit, sel), pp, keys);
                mark(0);
                ok = ok && bulk_barrier(Q, S, nbar);
                mark(1);
            }
            if (ok) ok = gemm_phase(Q, S, tiles, tmem, make_job(Q, G_PRED, 0, n_emit, sel), pp, keys);
            mark(2);
            ok = ok && bulk_barrier(Q, S, nbar);
            mark(3);
        }
        if (!ok) break;
        hidden_phase(Q, sel, n_live, n_prev);
        mark(4);
        if (!bulk_barrier(Q, S, nbar)) break;
        mark(5);
        if (!gemm_phase(Q, S, tiles, tmem, make_job(Q, G_JOINT, 0, n_live, sel), pp, keys)) break;
        mark(6);
        if (!bulk_barrier(Q, S, nbar)) break;
        mark(7);

        // ---- decision, part 1: this CTA's slice of the live list ----
        const int ch = (n_live + G - 1) / G;
        const int g = (int) blockIdx.x * ch + (int) threadIdx.x;
        const bool mine = (int) threadIdx.x < ch && g < n_live;
        const bool scr = screened(Q, n_live);
        if (scr) {                                      // exact argmax of the screened joint, a warp per row
            const Job JJ = make_job(Q, G_JOINT, 0, n_live, sel);
            for (int i = warp; i < ch && (int) blockIdx.x * ch + i < n_live; i += kBWarps) {
                int tk = 0, du = 0;
                screen_row(Q, JJ, (int) blockIdx.x * ch + i, tk, du);
                if ((threadIdx.x & 31) == 0) { S.tok_s[i] = tk; S.dur_s[i] = du; }
            }
            __syncthreads();
        }
        int e = 0, lv = 0, utt = -1, etok = 0, ereset = 0, ehb = 0, bad = 0;
        long long lframe = 0;
        if (mine) {
            utt = __ldcg(P.live + (size_t) sel * P.B + g);
            int * u = P.ust + utt * kUst;
            const unsigned long long kt = scr ? 0ull : __ldcg(&keys[2 * utt + 0]);
            const unsigned long long kd = (P.is_tdt && !scr) ? __ldcg(&keys[2 * utt + 1]) : 0ull;
            const int4 u0 = __ldcg(reinterpret_cast<const int4 *>(u));
            const int4 u1 = __ldcg(reinterpret_cast<const int4 *>(u) + 1);
            const int4 u2 = __ldcg(reinterpret_cast<const int4 *>(u) + 2);
            const long long foff = __ldg(P.frame_off + utt);
            const int uf[12] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w, u2.x, u2.y, u2.z, u2.w};
            int tok, di;
            bool kbad;
            if (scr) {
                tok = S.tok_s[threadIdx.x];
                di = S.dur_s[threadIdx.x];
                kbad = tok < 0 || tok >= P.V1 || (P.is_tdt && (di < 0 || di >= P.Nd));
            } else {
                keys[2 * utt + 0] = 0ull;
                if (P.is_tdt) keys[2 * utt + 1] = 0ull;
                tok = key_index(kt);
                di = P.is_tdt ? key_index(kd) : 0;
                kbad = keys_bad(P, kt, kd, tok, di);
            }
            if (kbad) {
                atomicCAS(&P.ctl[C_ERR], 0, (int) PK_ERR_DEVICE);
                P.ctl[C_ERRINFO] = utt;
                bad = 1;
                tok = P.blank;
                di = 0;
            }
            const int step = uf[U_STEPS];
            if (P.trace_steps > 0 && step < P.trace_steps) {
                const size_t ti = (size_t) utt * P.trace_steps + step;
                if (P.tr_tok) P.tr_tok[ti] = tok;
                if (P.tr_dur) P.tr_dur[ti] = di;
                if (P.forced_tok) {
                    const int ft = __ldg(P.forced_tok + ti);
                    if (ft >= 0 && ft < P.V1) {
                        tok = ft;
                        const int fd = P.forced_dur ? __ldg(P.forced_dur + ti) : 0;
                        di = (P.is_tdt && fd >= 0 && fd < P.Nd) ? fd : 0;
                    }
                }
            }
            u[U_STEPS] = step + 1;
            const int s0 = uf[U_SYM];
            const int T = uf[U_NFRAMES];
            const Decision d = decide_core(P, tok, di, s0);
            const int t = uf[U_T] + d.adv;
            e = d.e; etok = d.etok; ereset = d.ereset;
            int ntok = uf[U_NTOK];
            if (!P.is_tdt) eou_effects(P, u, uf, utt, d, s0, ntok, tok, T);
            if (d.emit_tok && !put_token(P, utt, tok, ntok, T)) bad = 1;
            if (e) {
                ehb = uf[U_HBUF] ^ 1;
                u[U_HBUF] = ehb;
            }
            u[U_T] = t;
            u[U_SYM] = d.sym;
            u[U_NTOK] = ntok;
            lv = t < T ? 1 : 0;
            if (lv) lframe = foff + t;
            if (!lv) P.finish_ns[utt] = gtimer();
        }
        int tot = 0;
        const int pf = bulk_scan(S, e | (lv << 16), tot);
        if (threadIdx.x == 0) Q.dcount[blockIdx.x] = make_int2(tot & 0xFFFF, tot >> 16);
        if (__syncthreads_or(bad)) { ok = false; break; }
        mark(8);
        if (!bulk_barrier(Q, S, nbar)) break;
        mark(9);

        // ---- decision, part 2: list positions from every CTA's counts ----
        int be = 0, bl = 0, te = 0, tl = 0;
        for (int k = threadIdx.x; k < G; k += blockDim.x) {
            const int2 c = __ldcg(Q.dcount + k);
            if (k < (int) blockIdx.x) { be += c.x; bl += c.y; }
            te += c.x;
            tl += c.y;
        }
        int sbe = 0, sbl = 0, ste = 0, stl = 0;
        bulk_scan(S, be, sbe);
        bulk_scan(S, bl, sbl);
        bulk_scan(S, te, ste);
        bulk_scan(S, tl, stl);
        const int nsel = sel ^ 1;
        if (scr && mine) Q.norm2[g] = 0.0f;        // read by part 1; the next hidden phase adds into it
        if (e) {
            reinterpret_cast<int2 *>(P.emit)[sbe + (pf & 0xFFFF)] =
                make_int2(utt, etok | (ehb << 30) | (ereset << 31));
        }
        if (lv) {
            const int pos = sbl + (pf >> 16);
            P.live[(size_t) nsel * P.B + pos] = utt;
            P.live_frame[(size_t) nsel * P.B + pos] = lframe;
            prefetch_l2(P.encp + (size_t) lframe * P.J, (unsigned) P.J * 4u);
        }
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            P.ctl[C_NEMIT] = ste;
            P.ctl[C_NLIVE0 + nsel] = stl;
            P.ctl[C_NDECIDED] = n_live;
            P.ctl[C_SEL] = nsel;
            P.ctl[C_ITERS] = iter + 1;
            P.ctl[C_EMITITERS] = emit_iters;
            P.ctl[C_BULKITERS] = iter + 1;
            P.ctl[C_BULKSTEPS] = (int) (sum_live + n_live);
            P.ctl[C_BULKEMITS] = (int) (sum_emit + n_emit);
            P.ctl[C_BULKSCREENED] = (int) (sum_scr + (scr ? n_live : 0));
        }
        sum_live += n_live;
        sum_emit += n_emit;
        if (scr) sum_scr += n_live;
        n_prev = n_live;
        sel = nsel;
        n_emit = ste;
        n_live = stl;
        ++iter;
        mark(10);
        if (!bulk_barrier(Q, S, nbar)) break;
        mark(11);
    }
    // hand the live utterances' state to the persistent loop (it reads its own layout)
    if (n_live + n_emit > 0 && __ldcg(&P.ctl[C_ERR]) == 0) handoff_phase(Q, sel, n_live, n_emit);
    if (prof) {
        for (int i = 0; i < 12; ++i) Q.prof[i] = pacc[i];
    }
    __syncthreads();
    if (prof)
        for (int i = 0; i < 8; ++i) Q.prof[12 + i] = S.rprof[i];

    // ---- teardown: every role is done with tensor memory ----
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 5) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// ---- bulk weights ------------------------------------------------------------------------

// dst [rows][K] hi / lo halves of row-gathered f32 weights: LSTM layer l uses
// rows 4j + q <- gate row q * H + j and K = [W_ih (kin) | W_hh (H)] (layer 0: W_hh only).
__global__ void bulk_split_lstm(const float * __restrict__ w_ih, const float * __restrict__ w_hh, int H, int kin,
                                __half * __restrict__ hi, __half * __restrict__ lo) {
    const int K = kin + H;
    const long long n = (long long) 4 * H * K;
    for (long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long) gridDim.x * blockDim.x) {
        const int r = (int) (i / K), k = (int) (i - (long long) r * K);
        const int j = r >> 2, q = r & 3;
        const int src = q * H + j;
        const float x = k < kin ? w_ih[(size_t) src * kin + k] : w_hh[(size_t) src * H + (k - kin)];
        const __half h = __float2half_rn(x);
        hi[i] = h;
        lo[i] = __float2half_rn(x - __half2float(h));
    }
}

__global__ void bulk_split_rows(const float * __restrict__ w, long long n, __half * __restrict__ hi,
                                __half * __restrict__ lo) {
    for (long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long) gridDim.x * blockDim.x) {
        const float x = w[i];
        const __half h = __float2half_rn(x);
        hi[i] = h;
        lo[i] = __float2half_rn(x - __half2float(h));
    }
}

__global__ void bulk_lstm_bias(const float * __restrict__ b_ih, const float * __restrict__ b_hh, int H,
                               float * __restrict__ out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= 4 * H) return;
    const int src = (r & 3) * H + (r >> 2);
    out[r] = b_ih[src] + b_hh[src];
}

// Embedding rows [V1][H] f32 -> rows of 4H bytes: f16 hi[H] | lo[H].
__global__ void bulk_split_embed(const float * __restrict__ e, long long n, int H, unsigned char * __restrict__ out) {
    for (long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long) gridDim.x * blockDim.x) {
        const long long v = i / H;
        const int j = (int) (i - v * H);
        const float x = e[i];
        const __half h = __float2half_rn(x);
        __half * row = reinterpret_cast<__half *>(out + v * 4LL * H);
        row[j] = h;
        row[H + j] = __float2half_rn(x - __half2float(h));
    }
}

// One row of a step-loop matrix requantised for the int8 path (one CTA per row): the
// row's values x, s = max|x| / 32639, W = round(x / s) split into signed digits
// W = 256 hi + lo (hi = floor((W + 128) / 256)), rscale = s. LSTM layers (lstm = 1)
// take row r = 4j + q from gate row q H + j with K = [W_ih (kin) | W_hh (H)] (kin = 0:
// W_hh only); otherwise row r of plain [N][K].
__global__ void bulk_i8_rows(const float * __restrict__ w_ih, const float * __restrict__ w_hh, int H, int kin,
                             int lstm, const float * __restrict__ plain, int K, signed char * __restrict__ hi,
                             signed char * __restrict__ lo, float * __restrict__ rscale) {
    __shared__ float red[32];
    const int r = blockIdx.x;
    const int src = lstm ? (r & 3) * H + (r >> 2) : r;
    auto val = [&](int k) -> float {
        if (!lstm) return plain[(size_t) r * K + k];
        return k < kin ? w_ih[(size_t) src * kin + k] : w_hh[(size_t) src * H + (k - kin)];
    };
    float m = 0.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, fabsf(val(k)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float x = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xFFFFFFFFu, x, o));
        if (threadIdx.x == 0) red[0] = x;
    }
    __syncthreads();
    const float sc = red[0] / 32639.0f;
    const float inv = sc > 0.0f ? 1.0f / sc : 0.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const int W = max(-32639, min(32639, __float2int_rn(val(k) * inv)));
        const int h = (W + 128) >> 8;
        hi[(size_t) r * K + k] = (signed char) h;
        lo[(size_t) r * K + k] = (signed char) (W - 256 * h);
    }
    if (threadIdx.x == 0) rscale[r] = sc;
}

// g0b[v][4j + q] = g0[v][q H + j] + b_hh0[q H + j] (g0 = b_ih0 + W_ih0 . embed[v]).
__global__ void bulk_g0_table(const float * __restrict__ g0, const float * __restrict__ b_hh0, int H, long long n,
                              float * __restrict__ out) {
    for (long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long) gridDim.x * blockDim.x) {
        const long long v = i / (4 * H);
        const int c = (int) (i - v * 4 * H);
        const int src = (c & 3) * H + (c >> 2);
        out[i] = g0[v * 4 * H + src] + b_hh0[src];
    }
}

// max over rows [0, rows) of ||w[r]||_2, rounded up (x 1.0001 covers the f32 sums for
// K <= 1024), into *out as float bits (positive floats order as unsigned integers).
__global__ void bulk_row_norm_max(const float * __restrict__ w, int rows, int K, unsigned * __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const long long nw = (long long) gridDim.x * blockDim.x / 32;
    for (long long r = ((long long) blockIdx.x * blockDim.x + threadIdx.x) / 32; r < rows; r += nw) {
        float ss = 0.0f;
        for (int k = lane; k < K; k += 32) {
            const float x = w[r * K + k];
            ss = fmaf(x, x, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
        if (lane == 0) atomicMax(out, __float_as_uint(sqrtf(ss) * 1.0001f));
    }
}

}  // namespace

cudaError_t encode_2d(void * map, CUtensorMapDataType type, size_t esize, const void * base, long long rows,
                      long long cols, int box_rows, int box_cols, CUtensorMapSwizzle swz);

bool bulk_supported(int H, int J, int L) {
    return H > 0 && J > 0 && H % kBK == 0 && J % kBK == 0 && L >= 1 && L <= kMaxLayers;
}

// TMA descriptor of `rows` activation rows of row_bytes bytes (a multiple of 16): bytes as
// elements, 128-row x 128-byte boxes, 128-byte swizzle (the bulk loop's A stage layout).
cudaError_t bulk_row_map(void * map, const void * base, long long rows, long long row_bytes) {
    return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, rows, row_bytes, kBM, 128, CU_TENSOR_MAP_SWIZZLE_128B);
}

// The same rows with 1-row boxes (tile::gather4 loads four arbitrary rows each).
cudaError_t bulk_row_map_gather(void * map, const void * base, long long rows, long long row_bytes) {
    return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, rows, row_bytes, 1, 128, CU_TENSOR_MAP_SWIZZLE_128B);
}

bool bulk_screen_supported(int J) { return J % 128 == 0 && J <= kScreenMaxJ; }

size_t bulk_smem_bytes() { return 1024 + (size_t) kRing + sizeof(BulkSmem); }

int bulk_threads() { return kBThreads; }

cudaError_t bulk_configure() {
    return cudaFuncSetAttribute(bulk_loop_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) bulk_smem_bytes());
}

cudaError_t bulk_occupancy(int * blocks_per_sm) {
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, bulk_loop_kernel, kBThreads, bulk_smem_bytes());
}

void bulk_release(BulkWeights & w) {
    if (w.mem) cudaFree(w.mem);
    w = BulkWeights{};
}

cudaError_t bulk_prepare(BulkWeights & w, int H, int J, int L, int Vo, int V1, const float * embed,
                         const float * const * w_ih, const float * const * w_hh, const float * const * b_ih,
                         const float * const * b_hh, const float * pred_w, const float * out_w,
                         const int * f16_weights, const float * g0, cudaStream_t s) {
    bulk_release(w);
    // the int8 LSTM / pred-proj path stages 128-element K blocks and splits layer K at H
    const bool i8 = g0 != nullptr && H % 128 == 0;
    // layout: [maps: (L + 2) x 2 x 128 B][row-norm bound, 256 B][lbias L x 4H f32][embedding halves]
    //         [weight halves]
    const int nmat = L + 2;
    size_t off = 0;
    const size_t maps = off;
    off += (size_t) nmat * 2 * 128;
    const size_t wn = off;
    off += 256;
    const size_t bias = off;
    off += (size_t) L * 4 * H * 4;
    off = (off + 255) & ~(size_t) 255;
    const size_t emb = off;
    off += (size_t) V1 * 4 * H;
    off = (off + 255) & ~(size_t) 255;
    size_t mat_off[kMaxLayers + 2];
    long long mat_rows[kMaxLayers + 2], mat_k[kMaxLayers + 2];
    for (int l = 0; l < L; ++l) { mat_rows[l] = 4LL * H; mat_k[l] = 2LL * H; }   // K = [W_ih | W_hh]
    mat_rows[L] = J; mat_k[L] = H;            // pred
    mat_rows[L + 1] = Vo; mat_k[L + 1] = J;   // joint
    for (int m = 0; m < nmat; ++m) {
        mat_off[m] = off;
        off += (size_t) 2 * mat_rows[m] * mat_k[m] * 2;
        off = (off + 255) & ~(size_t) 255;
    }
    // int8 path: [maps (L + 1) x 2 x 128 B][per matrix: hi, lo bytes, row scales (+128 pad)][g0b]
    const int nmi = L + 1;
    size_t imaps = 0, imat[kMaxLayers + 1] = {}, iscale[kMaxLayers + 1] = {}, g0b = 0;
    long long irows[kMaxLayers + 1] = {}, ik[kMaxLayers + 1] = {};
    if (i8) {
        imaps = off;
        off += (size_t) nmi * 2 * 128;
        for (int m = 0; m < nmi; ++m) {
            irows[m] = m < L ? 4LL * H : (long long) J;
            ik[m] = m < L ? (m == 0 ? (long long) H : 2LL * H) : (long long) H;
            off = (off + 255) & ~(size_t) 255;
            imat[m] = off;
            off += (size_t) 2 * irows[m] * ik[m];
            off = (off + 255) & ~(size_t) 255;
            iscale[m] = off;
            off += (size_t) (irows[m] + 128) * 4;
        }
        off = (off + 255) & ~(size_t) 255;
        g0b = off;
        off += (size_t) V1 * 4 * H * 4;
        off = (off + 255) & ~(size_t) 255;
    }
    cudaError_t e = cudaMalloc(&w.mem, off);
    if (e != cudaSuccess) { w.mem = nullptr; return e; }
    w.bytes = off;
    unsigned char * base = static_cast<unsigned char *>(w.mem);
    std::vector<CUtensorMap> host_maps((size_t) nmat * 2);   // 64-byte aligned, as the encoder requires
    for (int m = 0; m < nmat; ++m) {
        __half * hi = reinterpret_cast<__half *>(base + mat_off[m]);
        __half * lo = hi + mat_rows[m] * mat_k[m];
        if (m < L) {
            bulk_split_lstm<<<1184, 256, 0, s>>>(w_ih[m], w_hh[m], H, H, hi, lo);
        } else {
            bulk_split_rows<<<1184, 256, 0, s>>>(m == L ? pred_w : out_w, mat_rows[m] * mat_k[m], hi, lo);
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        e = encode_2d(&host_maps[(size_t) (2 * m)], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, hi, mat_rows[m],
                      mat_k[m], 64, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
        if (e != cudaSuccess) return e;
        e = encode_2d(&host_maps[(size_t) (2 * m + 1)], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, lo, mat_rows[m],
                      mat_k[m], 64, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
        if (e != cudaSuccess) return e;
        BulkGemm g;
        g.map_hi = base + maps + (size_t) (2 * m) * 128;
        g.map_lo = base + maps + (size_t) (2 * m + 1) * 128;
        g.hi = hi;
        g.lo = lo;
        g.N = (int) mat_rows[m];
        g.K = (int) mat_k[m];
        g.lo_zero = f16_weights[m];   // f16 weights are exact in the hi half
        if (m < L) w.gl[m] = g;
        else if (m == L) w.gp = g;
        else w.gj = g;
    }
    for (int l = 0; l < L; ++l) {
        bulk_lstm_bias<<<(4 * H + 255) / 256, 256, 0, s>>>(b_ih[l], b_hh[l], H,
                                                           reinterpret_cast<float *>(base + bias) + (size_t) l * 4 * H);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    bulk_split_embed<<<1184, 256, 0, s>>>(embed, (long long) V1 * H, H, base + emb);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(base + wn, 0, 256, s);
    if (e != cudaSuccess) return e;
    bulk_row_norm_max<<<1184, 256, 0, s>>>(out_w, V1, J, reinterpret_cast<unsigned *>(base + wn));
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    w.wnorm = reinterpret_cast<const float *>(base + wn);
    w.e16 = base + emb;
    w.lbias = reinterpret_cast<const float *>(base + bias);
    e = cudaMemcpyAsync(base + maps, host_maps.data(), host_maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return e;
    std::vector<CUtensorMap> imap_h((size_t) nmi * 2);   // (alive until the stream is synchronised)
    if (i8) {
        for (int m = 0; m < nmi; ++m) {
            signed char * hi = reinterpret_cast<signed char *>(base + imat[m]);
            signed char * lo = hi + irows[m] * ik[m];
            float * rs = reinterpret_cast<float *>(base + iscale[m]);
            e = cudaMemsetAsync(rs, 0, (size_t) (irows[m] + 128) * 4, s);
            if (e != cudaSuccess) return e;
            if (m < L)
                bulk_i8_rows<<<(unsigned) irows[m], 128, 0, s>>>(w_ih[m], w_hh[m], H, m == 0 ? 0 : H, 1, nullptr,
                                                                  (int) ik[m], hi, lo, rs);
            else
                bulk_i8_rows<<<(unsigned) irows[m], 128, 0, s>>>(nullptr, nullptr, H, 0, 0, pred_w, (int) ik[m], hi,
                                                                  lo, rs);
            e = cudaGetLastError();
            if (e != cudaSuccess) return e;
            e = encode_2d(&imap_h[(size_t) (2 * m)], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, hi, irows[m], ik[m], 64,
                          2 * kBK, CU_TENSOR_MAP_SWIZZLE_128B);
            if (e != cudaSuccess) return e;
            e = encode_2d(&imap_h[(size_t) (2 * m + 1)], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, lo, irows[m], ik[m], 64,
                          2 * kBK, CU_TENSOR_MAP_SWIZZLE_128B);
            if (e != cudaSuccess) return e;
            BulkGemm g{};
            g.map_hi = base + imaps + (size_t) (2 * m) * 128;
            g.map_lo = base + imaps + (size_t) (2 * m + 1) * 128;
            g.hi = hi;
            g.lo = lo;
            g.N = (int) irows[m];
            g.K = (int) ik[m];
            g.lo_zero = 0;
            g.i8 = 1;
            g.rscale = rs;
            if (m < L) w.gli[m] = g;
            else w.gpi = g;
        }
        bulk_g0_table<<<1184, 256, 0, s>>>(g0, b_hh[0], H, (long long) V1 * 4 * H, reinterpret_cast<float *>(base + g0b));
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        w.g0b = reinterpret_cast<const float *>(base + g0b);
        e = cudaMemcpyAsync(base + imaps, imap_h.data(), imap_h.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return e;
        w.i8_ok = 1;
    }
    return cudaStreamSynchronize(s);
}

cudaError_t launch_bulk(const BulkParams & q, int grid, cudaStream_t s) {
    void * args[] = {const_cast<BulkParams *>(&q)};
    return cudaLaunchCooperativeKernel(reinterpret_cast<const void *>(bulk_loop_kernel), dim3(grid), dim3(kBThreads),
                                       args, bulk_smem_bytes(), s);
}

}  // namespace pk
