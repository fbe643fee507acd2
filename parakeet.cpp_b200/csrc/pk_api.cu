// pk_api.cu -- the extern "C" surface of libparakeet_cuda (include/parakeet_cuda.h):
// context creation and weight repack, the per-call workspace, and the batch,
// trace and streaming entry points built on the persistent step loop.

#include "pk_internal.h"

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

namespace {

thread_local std::string g_err;

pk_status fail(pk_status s, const char * fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return s;
}

#define PK_CK(call)                                                                         \
    do {                                                                                    \
        cudaError_t e_ = (call);                                                            \
        if (e_ != cudaSuccess)                                                              \
            return fail(e_ == cudaErrorMemoryAllocation ? PK_ERR_OOM : PK_ERR_CUDA,         \
                        "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
    } while (0)

#define PK_TRY(expr)                      \
    do {                                  \
        pk_status s_ = (expr);            \
        if (s_ != PK_OK) return s_;       \
    } while (0)

struct DevBuf {
    void * p = nullptr;
    size_t cap = 0;
    cudaError_t ensure(size_t bytes) {
        if (bytes <= cap && (p != nullptr || bytes == 0)) return cudaSuccess;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        const size_t want = bytes + bytes / 8 + 256;
        cudaError_t e = cudaMalloc(&p, want);
        if (e == cudaSuccess) cap = want;
        return e;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
    }
    template <class T> T * as() const { return static_cast<T *>(p); }
};

}  // namespace

struct pk_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    int sm_count = 0, grid = 0, chunk = 32, ldx = 0;
    size_t smem = 0;
    int type = PK_MODEL_TDT, H = 0, J = 0, De = 0, L = 0, V = 0, V1 = 0, Vo = 0, Nd = 0;
    int blank = 0, eou = -1, eob = -1, max_sym = 10, n_special = 0;
    long long timeout_ns = 5000000000ll;
    int math = PK_MATH_F32;
    int test_stall = 0;
    // tensor-core step loop
    int tc_ok = 0, tc_stationary = 0, rpc_j = 0, rpc_p = 0, upc = 0, tc_hint = 0;
    int tc_rbh = 0, tc_rbj = 0;   // staged row bytes: h, hid
    int tc_area = 0, tc_mb = 1;   // shared-memory staging area bytes, m16 blocks per pass
    unsigned tc_sm_weights = 0;
    size_t tc_smem = 0;
    pk::TcBlock tcj{}, tcp{}, tcl[pk::kMaxLayers]{};
    DevBuf tc_frag[2 + pk::kMaxLayers], tc_scale[2 + pk::kMaxLayers], g0;
    uint64_t weight_bytes = 0;
    // tensor-core enc-proj: f16 hi / lo weights and their TMA descriptor
    int ep_ok = 0;
    DevBuf ep_w16, ep_err;
    alignas(64) unsigned char ep_tmap[128] = {};
    // weights (f32 on the device)
    DevBuf embed, w_ih[pk::kMaxLayers], w_hh[pk::kMaxLayers], b_ih[pk::kMaxLayers],
        b_hh[pk::kMaxLayers], enc_w, enc_b, pred_w, pred_b, out_w, out_b, durations, special;
    // bulk loop (tcgen05, many live utterances): weights, threshold, per-call buffers
    pk::BulkWeights bulk{};
    int bulk_ok = 0;
    int bulk_min_live = 128;
    int bulk_screen_min = 1024;    // PK_OPT_BULK_SCREEN
    int bulk_i8 = 1;               // PK_OPT_BULK_I8
    int bulk_tma_a = 1;            // PK_OPT_BULK_TMA_A
    DevBuf h16, x16, dcount, bprof, norm2, jsum;
    void * pin = nullptr;          // pinned staging of a call's small inputs (copy_segments)
    size_t pin_cap = 0;
    // per-call workspace
    DevBuf prof;
    DevBuf livef, hst, xnew, hidc;
    DevBuf enc, encp, h, c, predp, hid, ust, keys, live, emit, ctl, bar, tstart, finish, tok,
        tokregion, bnd, bndregion, frameoff, offsets, boffsets, compact, bcompact;
    DevBuf tr_logits, tr_h, tr_c, tr_tok, tr_dur, tr_ftok, tr_fdur;
    cudaEvent_t ev[7] = {};
    // prefetched host encoder outputs: up to two staged copies made on a copy stream
    // (pk_prefetch_batch), each named by its ticket n + 1; copy n records cev[n & 1]
    cudaStream_t cstream = nullptr;
    cudaEvent_t cev[2] = {};
    uint64_t n_copies = 0;
    DevBuf stg[2];
    int64_t stg_frames[2] = {0, 0};
    uint64_t stg_seq[2] = {0, 0};   // 0: empty; else 1 + the copy's number = its ticket
    std::vector<DevBuf *> all_bufs() {
        std::vector<DevBuf *> v = {&embed, &enc_w, &enc_b, &pred_w, &pred_b, &out_w, &out_b,
                                   &durations, &special, &enc, &encp, &h, &c, &predp, &hid, &ust,
                                   &keys, &live, &emit, &ctl, &bar, &tstart, &finish, &tok,
                                   &tokregion, &bnd, &bndregion, &frameoff, &offsets, &boffsets,
                                   &compact, &bcompact, &tr_logits, &tr_h, &tr_c, &tr_tok, &tr_dur,
                                   &tr_ftok, &tr_fdur, &g0, &prof, &livef, &hst, &xnew, &hidc, &ep_w16, &ep_err, &h16, &x16, &dcount, &bprof,
                                   &norm2, &jsum, &stg[0], &stg[1]};
        for (int i = 0; i < 2 + pk::kMaxLayers; ++i) { v.push_back(&tc_frag[i]); v.push_back(&tc_scale[i]); }
        for (int l = 0; l < pk::kMaxLayers; ++l) {
            v.push_back(&w_ih[l]); v.push_back(&w_hh[l]); v.push_back(&b_ih[l]); v.push_back(&b_hh[l]);
        }
        return v;
    }
};

struct pk_stream {
    pk_ctx * ctx = nullptr;
    DevBuf h, c;     // [L][H]
    int sym = 0, carry = 0, initialized = 0, last = -1, segstart = 0, symx = 0;
};

namespace {

using namespace pk;

bool shape_ok(const pk_tensor & t, int64_t ne0, int64_t ne1) {
    return t.data && t.ne0 == ne0 && (ne1 <= 1 ? (t.ne1 <= 1) : t.ne1 == ne1);
}

// Every copy goes through the context's stream (a non-blocking stream does not
// order against the legacy default stream that plain cudaMemcpy/cudaMemset use:
// a pageable host->device cudaMemcpy may return before its DMA lands).
cudaError_t copy_sync(pk_ctx * x, void * dst, const void * src, size_t n, cudaMemcpyKind kind) {
    if (n == 0) return cudaSuccess;
    cudaError_t e = cudaMemcpyAsync(dst, src, n, kind, x->stream);
    if (e != cudaSuccess) return e;
    return cudaStreamSynchronize(x->stream);
}

size_t raw_bytes(int type, int64_t ne0, int64_t rows) {
    if (type == PK_GGML_F32) return (size_t) (ne0 * rows) * 4;
    if (type == PK_GGML_F16) return (size_t) (ne0 * rows) * 2;
    return (size_t) (rows * (ne0 / 32)) * 34;
}

// Upload one GGUF tensor (first `keep_rows` rows) and dequantize it to f32.
pk_status upload(pk_ctx * x, const pk_tensor & t, int64_t keep_rows, DevBuf & dst, DevBuf & scratch,
                 const char * name) {
    if (!t.data) return fail(PK_ERR_MODEL, "tensor %s missing", name);
    if (t.type != PK_GGML_F32 && t.type != PK_GGML_F16 && t.type != PK_GGML_Q8_0)
        return fail(PK_ERR_MODEL, "tensor %s: unsupported ggml type %d", name, t.type);
    if (t.type == PK_GGML_Q8_0 && t.ne0 % 32 != 0)
        return fail(PK_ERR_MODEL, "tensor %s: q8_0 row of %lld not a multiple of 32", name, (long long) t.ne0);
    const int64_t rows_all = t.ne1 > 0 ? t.ne1 : 1;
    const int64_t rows = std::min(rows_all, keep_rows);
    const size_t nb = raw_bytes(t.type, t.ne0, rows);
    if (t.nbytes < nb) return fail(PK_ERR_MODEL, "tensor %s: %llu bytes < %zu needed", name,
                                   (unsigned long long) t.nbytes, nb);
    PK_CK(scratch.ensure(nb));
    PK_CK(cudaMemcpyAsync(scratch.p, t.data, nb, cudaMemcpyHostToDevice, x->stream));
    const size_t fb = (size_t) (t.ne0 * rows) * sizeof(float);
    PK_CK(dst.ensure(fb));
    PK_CK(launch_dequant(scratch.p, t.type, t.ne0, rows, dst.as<float>(), x->stream));
    PK_CK(cudaStreamSynchronize(x->stream));
    x->weight_bytes += fb;
    return PK_OK;
}

// ---- tensor-core weight repack (host side, once at pk_create) ----------------

float half_bits_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int sh = 0;
            while ((m & 0x400u) == 0) { m <<= 1; ++sh; }
            bits = sign | ((uint32_t) (113 - sh) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// A weight matrix as seen by one phase: rows of tensor `a`, optionally
// continued along K by tensor `b` (the [W_ih | W_hh] concatenation).
struct SrcMat {
    const pk_tensor * a = nullptr;
    const pk_tensor * b = nullptr;
    int64_t ka = 0;
    int type() const { return a->type; }
    const pk_tensor & at(int64_t k, int64_t & kk) const {
        if (b && k >= ka) { kk = k - ka; return *b; }
        kk = k;
        return *a;
    }
    int8_t q(int64_t row, int64_t k) const {
        int64_t kk;
        const pk_tensor & t = at(k, kk);
        const uint8_t * blk = static_cast<const uint8_t *>(t.data) + (row * (t.ne0 / 32) + kk / 32) * 34;
        return (int8_t) blk[2 + kk % 32];
    }
    uint8_t q_biased(int64_t row, int64_t k) const {
        int64_t kk;
        const pk_tensor & t = at(k, kk);
        const uint8_t * blk = static_cast<const uint8_t *>(t.data) + (row * (t.ne0 / 32) + kk / 32) * 34;
        return (uint8_t) ((int) (int8_t) blk[2 + kk % 32] + 128);
    }
    float scale(int64_t row, int64_t k) const {
        int64_t kk;
        const pk_tensor & t = at(k, kk);
        const uint8_t * blk = static_cast<const uint8_t *>(t.data) + (row * (t.ne0 / 32) + kk / 32) * 34;
        return half_bits_to_float((uint16_t) (blk[0] | (blk[1] << 8)));
    }
    uint16_t half(int64_t row, int64_t k) const {
        int64_t kk;
        const pk_tensor & t = at(k, kk);
        return static_cast<const uint16_t *>(t.data)[row * t.ne0 + kk];
    }
};

// imma: q8_0 rows packed as raw int8 B fragments of mma.m16n8k32 (lane (g, t):
// k = 4t..4t+3 then 16+4t..16+4t+3 of each 32-wide block); otherwise f16
// fragments of mma.m16n8k16 (q8_0 stored q + 128, converted exactly in-kernel).
template <class RowMap>
pk_status build_tc_block(pk_ctx * x, int G, int tiles, int K, const SrcMat & src, RowMap rowmap,
                         DevBuf & dfrag, DevBuf & dscale, pk::TcBlock & out, bool imma = false) {
    const bool i8 = src.type() == PK_GGML_Q8_0;
    imma = imma && i8;
    const int nkb = K / 32;
    const size_t per_lane = i8 ? 8 : 16;
    const size_t cta_bytes = (size_t) tiles * nkb * 32 * per_lane;
    const size_t cta_scales = i8 ? (size_t) tiles * nkb * 8 : 0;
    std::vector<uint8_t> frag((size_t) G * cta_bytes);
    std::vector<float> scale(std::max<size_t>((size_t) G * cta_scales, 1), 0.0f);
    for (int cta = 0; cta < G; ++cta) {
        for (int tile = 0; tile < tiles; ++tile) {
            for (int kb = 0; kb < nkb; ++kb) {
                for (int lane = 0; lane < 32; ++lane) {
                    const int g = lane >> 2, t = lane & 3;
                    const int64_t row = rowmap(cta, tile * 8 + g);
                    uint8_t * dst = frag.data() + (size_t) cta * cta_bytes +
                                    (((size_t) tile * nkb + kb) * 32 + lane) * per_lane;
                    if (imma) {
                        for (int e = 0; e < 8; ++e) {
                            const int64_t k = (int64_t) kb * 32 + (e < 4 ? 4 * t + e : 16 + 4 * t + e - 4);
                            dst[e] = row < 0 ? (uint8_t) 0 : (uint8_t) src.q(row, k);
                        }
                        continue;
                    }
                    for (int ks = 0; ks < 2; ++ks) {
                        const int64_t kk = (int64_t) kb * 32 + ks * 16;
                        const int64_t ks4[4] = {kk + 2 * t, kk + 2 * t + 1, kk + 2 * t + 8, kk + 2 * t + 9};
                        for (int e = 0; e < 4; ++e) {
                            if (i8) {
                                dst[ks * 4 + e] = row < 0 ? (uint8_t) 128 : src.q_biased(row, ks4[e]);
                            } else {
                                const uint16_t hv = row < 0 ? (uint16_t) 0 : src.half(row, ks4[e]);
                                std::memcpy(dst + (ks * 4 + e) * 2, &hv, 2);
                            }
                        }
                    }
                }
                if (i8) {
                    for (int rr = 0; rr < 8; ++rr) {
                        const int64_t row = rowmap(cta, tile * 8 + rr);
                        scale[(size_t) cta * cta_scales + ((size_t) tile * nkb + kb) * 8 + rr] =
                            row < 0 ? 0.0f : src.scale(row, (int64_t) kb * 32);
                    }
                }
            }
        }
    }
    PK_CK(dfrag.ensure(frag.size()));
    PK_CK(copy_sync(x, dfrag.p, frag.data(), frag.size(), cudaMemcpyHostToDevice));
    PK_CK(dscale.ensure(scale.size() * 4));
    PK_CK(copy_sync(x, dscale.p, scale.data(), scale.size() * 4, cudaMemcpyHostToDevice));
    out.frag = dfrag.as<uint8_t>();
    out.scale = dscale.as<float>();
    out.cta_bytes = (unsigned) cta_bytes;
    out.cta_scales = (unsigned) cta_scales;
    out.tiles = tiles;
    out.K = K;
    out.is_i8 = i8 ? 1 : 0;
    out.imma = imma ? 1 : 0;
    return PK_OK;
}

bool tc_type_ok(const pk_tensor & t) { return t.type == PK_GGML_Q8_0 || t.type == PK_GGML_F16; }

// Repack the step-loop weights for the tensor-core phases; leaves x->tc_ok = 0
// (CUDA-core f32 phases only) when the model does not qualify.
pk_status setup_tc(pk_ctx * x, const pk_model_desc * d, size_t smem_cap) {
    const int H = x->H, J = x->J, L = x->L, G = x->grid;
    x->tc_ok = 0;
    if (H % 32 != 0 || J % 32 != 0) return PK_OK;
    if (!tc_type_ok(d->joint_out_w) || !tc_type_ok(d->joint_pred_w) || !tc_type_ok(d->lstm[0].w_hh)) return PK_OK;
    for (int l = 1; l < L; ++l)
        if (!tc_type_ok(d->lstm[l].w_ih) || d->lstm[l].w_ih.type != d->lstm[l].w_hh.type) return PK_OK;
    // int16 activations on int8 tensor cores when every LSTM / pred-proj weight is q8_0
    bool all_q8 = d->joint_pred_w.type == PK_GGML_Q8_0 && d->lstm[0].w_hh.type == PK_GGML_Q8_0;
    for (int l = 1; l < L; ++l) all_q8 = all_q8 && d->lstm[l].w_ih.type == PK_GGML_Q8_0;
    x->tc_hint = all_q8 ? 1 : 0;
    x->rpc_j = (x->Vo + G - 1) / G;
    x->rpc_p = (J + G - 1) / G;
    x->upc = (H + G - 1) / G;
    const int rpc_j = x->rpc_j, rpc_p = x->rpc_p, upc = x->upc, Vo = x->Vo;
    SrcMat sj; sj.a = &d->joint_out_w;
    PK_TRY(build_tc_block(x, G, (rpc_j + 7) / 8, J, sj,
                          [&](int cta, int r) -> int64_t {
                              const int64_t row = (int64_t) cta * rpc_j + r;
                              return (r < rpc_j && row < Vo) ? row : -1; },
                          x->tc_frag[0], x->tc_scale[0], x->tcj));
    SrcMat sp; sp.a = &d->joint_pred_w;
    PK_TRY(build_tc_block(x, G, (rpc_p + 7) / 8, H, sp,
                          [&](int cta, int r) -> int64_t {
                              const int64_t row = (int64_t) cta * rpc_p + r;
                              return (r < rpc_p && row < J) ? row : -1; },
                          x->tc_frag[1], x->tc_scale[1], x->tcp, x->tc_hint != 0));
    auto unit_rows = [&](int cta, int r) -> int64_t {
        const int jj = r / 4, q = r % 4;
        const int64_t unit = (int64_t) cta * upc + jj;
        return (jj < upc && unit < H) ? (int64_t) q * H + unit : -1;
    };
    const int tiles_l = (4 * upc + 7) / 8;
    if (tiles_l > kTcRmax) return PK_OK;      // the LSTM phase runs one GEMM group per CTA
    for (int l = 0; l < L; ++l) {
        SrcMat sl;
        if (l == 0) {
            sl.a = &d->lstm[0].w_hh;                       // W_ih0 . embed comes from the g0 table
        } else {
            sl.a = &d->lstm[l].w_ih; sl.b = &d->lstm[l].w_hh; sl.ka = H;
        }
        PK_TRY(build_tc_block(x, G, tiles_l, l == 0 ? H : 2 * H, sl, unit_rows,
                              x->tc_frag[2 + l], x->tc_scale[2 + l], x->tcl[l], x->tc_hint != 0));
    }
    // g0[v][4H] = b_ih0 + W_ih0 . embed[v] for every token v (f32 GEMM on the device)
    PK_CK(x->g0.ensure((size_t) x->V1 * 4 * H * 4));
    PK_CK(launch_encproj_f32(x->embed.as<float>(), x->V1, H, x->w_ih[0].as<float>(), x->b_ih[0].as<float>(),
                             4 * H, x->g0.as<float>(), x->stream));
    PK_CK(cudaStreamSynchronize(x->stream));
    // stationary shared-memory layout
    unsigned off = 0;
    auto place = [&](pk::TcBlock & b) {
        b.sm_frag = off; off += (b.cta_bytes + 15u) & ~15u;
        b.sm_scale = off; off += ((b.cta_scales * 4u) + 15u) & ~15u;
    };
    place(x->tcj);
    place(x->tcp);
    for (int l = 0; l < L; ++l) place(x->tcl[l]);
    // staged rows: [hi | lo] + 16 bytes, an odd multiple of 16 (conflict-free ldmatrix rows)
    x->tc_rbh = 2 * H * (x->tc_hint ? 1 : 2) + 16;
    x->tc_rbj = 4 * J + 16;
    // staging area for a pass of 16 * mb utterances: the joint hidden rows, or the
    // LSTM's one or two h segments, or afterwards the GEMM's per-warp partial sums
    auto area_for = [&](int mb) -> int {
        const size_t pr = (size_t) kTcM * mb;
        const size_t part = (size_t) kWarps * (mb == 2 ? 7 : kTcRmax) * 8 * (pr + 4) * 4;   // rows padded by 4
        // a joint or pred-proj slice of more tiles than one GEMM call takes is done
        // call by call on one staged tile: its partial sums (and the argmax keys) go after it
        const int tg = mb == 2 ? 7 : kTcRmax;
        const size_t jkeep = x->tcj.tiles <= tg ? 0
            : pr * x->tc_rbj + std::max<size_t>((size_t) 4 * tg * 8 * (pr + 4) * 4, kThreads * 16) + 16;
        const size_t pkeep = x->tcp.tiles <= tg ? 0
            : pr * x->tc_rbh + std::max<size_t>((size_t) (mb == 2 ? kWarps : 4) * tg * 8 * (pr + 4) * 4,
                                                kThreads * 16) + 16;
        const size_t a = std::max({pr * x->tc_rbj, (L > 1 ? 2 : 1) * pr * x->tc_rbh, part, jkeep, pkeep});
        return (int) ((a + 15) & ~(size_t) 15);
    };
    // passes of 32 when the LSTM slice fits one two-block GEMM call (7 tiles) and
    // 32 utterances x the CTA's units fit one thread each in the cell update
    const bool mb2_ok = tiles_l <= 7 && kTcM * 2 * upc <= kThreads;   // one call per LSTM pass
    size_t need = 0;
    x->tc_stationary = 0;
    for (int mb = mb2_ok ? 2 : 1; mb >= 1 && !x->tc_stationary; --mb) {
        need = step_loop_tc_smem_bytes(off, area_for(mb), rpc_j, rpc_p, upc);
        if (need <= smem_cap) {
            x->tc_stationary = 1;
            x->tc_sm_weights = off;
            x->tc_mb = mb;
            x->tc_area = area_for(mb);
        }
    }
    if (!x->tc_stationary) {
        x->tc_sm_weights = 0;
        x->tc_mb = 1;
        x->tc_area = area_for(1);
        need = step_loop_tc_smem_bytes(0, x->tc_area, rpc_j, rpc_p, upc);
        if (need > smem_cap) return PK_OK;
    }
    x->tc_smem = need;
    if (step_loop_configure(x->tc_smem, 1) != cudaSuccess) return PK_OK;
    int per_sm = 0;
    if (step_loop_occupancy(x->tc_smem, 1, &per_sm) != cudaSuccess || per_sm < 1) return PK_OK;
    x->tc_ok = 1;
    return PK_OK;
}

// Tensor-core enc-proj (f16 hi / lo weights + TMA descriptor); leaves ep_ok = 0
// (CUDA-core f32 enc-proj) when the shapes or the device do not allow it.
void setup_encproj(pk_ctx * x, size_t smem_cap) {
    x->ep_ok = 0;
    if (!encproj_tc_supported(x->De, x->J) || encproj_tc_smem_bytes() > smem_cap) return;
    if (x->ep_w16.ensure((size_t) 2 * x->J * x->De * 2) != cudaSuccess) return;
    if (x->ep_err.ensure(sizeof(int)) != cudaSuccess) return;
    if (cudaMemsetAsync(x->ep_err.p, 0, sizeof(int), x->stream) != cudaSuccess) return;
    if (encproj_tc_prepare(x->enc_w.as<float>(), x->J, x->De, x->ep_w16.as<unsigned short>(), x->ep_tmap,
                           x->stream) != cudaSuccess) return;
    if (encproj_tc_configure() != cudaSuccess) return;
    if (cudaStreamSynchronize(x->stream) != cudaSuccess) return;
    x->ep_ok = 1;
}

pk_status validate_desc(const pk_model_desc * d) {
    if (!d) return fail(PK_ERR_INVALID, "null descriptor");
    if (d->model_type != PK_MODEL_TDT && d->model_type != PK_MODEL_EOU)
        return fail(PK_ERR_MODEL, "bad model_type %d", d->model_type);
    const int H = d->pred_hidden, J = d->joint_hidden, De = d->d_enc, L = d->n_layers;
    const int V1 = d->vocab_size + 1;
    if (H <= 0 || J <= 0 || De <= 0 || L <= 0 || d->vocab_size <= 0)
        return fail(PK_ERR_MODEL, "bad dims H=%d J=%d De=%d L=%d V=%d", H, J, De, L, d->vocab_size);
    if (L > kMaxLayers) return fail(PK_ERR_MODEL, "%d LSTM layers > %d supported", L, kMaxLayers);
    if (H % 4 != 0 || J % 4 != 0)
        return fail(PK_ERR_MODEL, "pred_hidden and joint_hidden must be multiples of 4");
    if (d->blank_id < 0 || d->blank_id >= V1) return fail(PK_ERR_MODEL, "blank_id out of range");
    const int Nd = d->model_type == PK_MODEL_TDT ? d->num_durations : 0;
    if (d->model_type == PK_MODEL_TDT) {
        if (Nd <= 0 || !d->durations) return fail(PK_ERR_MODEL, "TDT model needs durations");
        for (int i = 0; i < Nd; ++i)
            if (d->durations[i] < 0) return fail(PK_ERR_MODEL, "negative duration");
    }
    const int Vo = V1 + Nd;
    if (!d->lstm) return fail(PK_ERR_MODEL, "missing LSTM layers");
    if (d->embed.ne0 != H || d->embed.ne1 < V1) return fail(PK_ERR_MODEL, "embed shape");
    if (!shape_ok(d->joint_enc_w, De, J) || !shape_ok(d->joint_enc_b, J, 1))
        return fail(PK_ERR_MODEL, "joint.enc shape");
    if (!shape_ok(d->joint_pred_w, H, J) || !shape_ok(d->joint_pred_b, J, 1))
        return fail(PK_ERR_MODEL, "joint.pred shape");
    if (d->joint_out_w.ne0 != J || d->joint_out_w.ne1 < Vo || d->joint_out_b.ne0 < Vo)
        return fail(PK_ERR_MODEL, "joint.out shape");
    for (int l = 0; l < L; ++l) {
        const pk_lstm_layer & y = d->lstm[l];
        if (!shape_ok(y.w_ih, H, 4 * H) || !shape_ok(y.w_hh, H, 4 * H) ||
            !shape_ok(y.b_ih, 4 * H, 1) || !shape_ok(y.b_hh, 4 * H, 1))
            return fail(PK_ERR_MODEL, "lstm layer %d shape", l);
    }
    return PK_OK;
}

// Arguments of one run of the step loop.
struct Run {
    const float * enc = nullptr;
    bool enc_dev = false;
    int B = 0;
    const int64_t * frame_off = nullptr;
    const int32_t * n_frames = nullptr;
    int msym = 1;
    uint64_t ticket = 0;             // staged prefetch copy to read (pk_batch::prefetch_ticket)
    std::vector<int32_t> t0, sym0, nbefore, segstart, last, symx, fresh;
    const float * h_in = nullptr;    // device [L][H] state to resume (B == 1)
    const float * c_in = nullptr;
    const pk_trace * trace = nullptr;
    // outputs
    std::vector<int32_t> ust;
    std::vector<int32_t> ctl;
    unsigned long long prof[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    unsigned long long bprof[20] = {};
    float ms_encproj = 0.f, ms_loop = 0.f, ms_bulk = 0.f;
    int launches = 0;          // kernels launched by this call
};

pk_status run_loop(pk_ctx * x, Run & r) {
    const int B = r.B, H = x->H, J = x->J, L = x->L;
    cudaStream_t s = x->stream;
    // the loop's control word carries live and emit counts in 23 bits each
    if (B >= (1 << 23)) return fail(PK_ERR_INVALID, "batch of %d utterances exceeds %d", B, (1 << 23) - 1);
    int64_t frames = 0;
    for (int b = 0; b < B; ++b) {
        if (r.n_frames[b] < 0) return fail(PK_ERR_INVALID, "n_frames[%d] < 0", b);
        if (r.n_frames[b] > 0) {
            if (r.frame_off[b] < 0) return fail(PK_ERR_INVALID, "frame_offsets[%d] < 0", b);
            frames = std::max<int64_t>(frames, r.frame_off[b] + r.n_frames[b]);
        }
    }
    int stage = -1;                  // the staged prefetch copy this call reads
    if (r.ticket) {
        if (r.enc_dev) return fail(PK_ERR_INVALID, "prefetch_ticket given with device input");
        for (int i = 0; i < 2; ++i)
            if (x->stg_seq[i] == r.ticket) stage = i;
        if (stage < 0)
            return fail(PK_ERR_INVALID, "prefetch ticket %llu is not staged (already used, or replaced "
                        "by two later prefetches)", (unsigned long long) r.ticket);
        if (x->stg_frames[stage] < frames)
            return fail(PK_ERR_INVALID, "prefetch ticket %llu holds %lld frames, the batch reads %lld",
                        (unsigned long long) r.ticket, (long long) x->stg_frames[stage], (long long) frames);
    }
    if (frames > 0 && !r.enc && stage < 0) return fail(PK_ERR_INVALID, "null encoder output");
    const int msym1 = std::max(1, r.msym);
    std::vector<int64_t> tokregion(B), bndregion(B);
    int64_t tok_total = 0, bnd_total = 0;
    for (int b = 0; b < B; ++b) {
        tokregion[b] = tok_total;
        bndregion[b] = bnd_total;
        tok_total += (int64_t) r.n_frames[b] * msym1;
        bnd_total += r.n_frames[b];
    }
    const size_t Bs = (size_t) std::max(B, 1);
    PK_CK(x->encp.ensure((size_t) frames * J * 4));
    PK_CK(x->h.ensure(2 * (size_t) L * Bs * H * 4));
    PK_CK(x->c.ensure((size_t) L * Bs * H * 4));
    const bool use_tc = (x->math == PK_MATH_TC || x->math == PK_MATH_Q8) && x->tc_ok;
    if (use_tc) {
        PK_CK(x->hst.ensure(2 * (size_t) L * Bs * x->tc_rbh));
        PK_CK(x->xnew.ensure((size_t) L * Bs * x->tc_rbh));
        PK_CK(x->hidc.ensure((size_t) Bs * x->tc_rbj));
    }
    PK_CK(x->predp.ensure(Bs * J * 4));
    PK_CK(x->hid.ensure(Bs * J * 4));
    PK_CK(x->ust.ensure(Bs * kUst * 4));
    PK_CK(x->keys.ensure(Bs * 4 * 8));   // two alternating [B][2] argmax key buffers
    PK_CK(x->live.ensure(2 * Bs * 4));
    PK_CK(x->livef.ensure(2 * Bs * 8));
    PK_CK(x->emit.ensure(2 * Bs * 4));
    PK_CK(x->ctl.ensure(kCtl * 4));
    PK_CK(x->bar.ensure(8 * 4));
    PK_CK(x->tstart.ensure(8));
    PK_CK(x->prof.ensure(8 * 8));
    PK_CK(cudaMemsetAsync(x->prof.p, 0, 8 * 8, x->stream));
    PK_CK(x->finish.ensure(Bs * 8));
    PK_CK(x->tok.ensure((size_t) std::max<int64_t>(tok_total, 1) * 4));
    PK_CK(x->tokregion.ensure(Bs * 8));
    PK_CK(x->bnd.ensure((size_t) std::max<int64_t>(bnd_total, 1) * 4));
    PK_CK(x->bndregion.ensure(Bs * 8));
    PK_CK(x->frameoff.ensure(Bs * 8));

    PK_CK(cudaEventRecord(x->ev[0], s));
    const float * encsrc = r.enc;
    if (stage >= 0) {
        // the prefetched copy: the device waits for it (copy n recorded cev[n & 1]; a
        // later copy that re-recorded that event was queued after it on the copy stream)
        PK_CK(cudaStreamWaitEvent(s, x->cev[(x->stg_seq[stage] - 1) & 1], 0));
        encsrc = x->stg[stage].as<float>();
        x->stg_seq[stage] = 0;       // a ticket is used once
    } else if (frames > 0 && !r.enc_dev) {
        PK_CK(x->enc.ensure((size_t) frames * x->De * 4));
        PK_CK(cudaMemcpyAsync(x->enc.p, r.enc, (size_t) frames * x->De * 4, cudaMemcpyHostToDevice, s));
        encsrc = x->enc.as<float>();
    }
    PK_CK(cudaEventRecord(x->ev[1], s));
    const bool ep_tc = use_tc && x->ep_ok && (reinterpret_cast<uintptr_t>(encsrc) & 15u) == 0;
    if (frames > 0) {
        if (ep_tc)
            PK_CK(launch_encproj_tc(encsrc, frames, x->De, x->ep_tmap, J, x->enc_b.as<float>(), x->encp.as<float>(),
                                    x->timeout_ns, x->ep_err.as<int>(), s));
        else
            PK_CK(launch_encproj_f32(encsrc, frames, x->De, x->enc_w.as<float>(), x->enc_b.as<float>(), J,
                                     x->encp.as<float>(), s));
        ++r.launches;
    }
    PK_CK(cudaEventRecord(x->ev[2], s));

    // Host-built initial per-utterance state and lists.
    std::vector<int32_t> ust((size_t) B * kUst, 0), live, emit;
    std::vector<int64_t> live_frame;
    for (int b = 0; b < B; ++b) {
        int32_t * u = &ust[(size_t) b * kUst];
        u[U_T] = r.t0[b];
        u[U_SYM] = r.sym0[b];
        u[U_HBUF] = 0;
        u[U_LAST] = r.last[b];
        u[U_SEGSTART] = r.segstart[b];
        u[U_NBEFORE] = r.nbefore[b];
        u[U_NFRAMES] = r.n_frames[b];
        u[U_SYMX] = r.symx[b];
        if (r.n_frames[b] > 0 && r.t0[b] < r.n_frames[b]) {
            live.push_back(b);
            live_frame.push_back(r.frame_off[b] + r.t0[b]);
        }
        if (r.fresh[b]) { emit.push_back(b); emit.push_back(x->blank | (1 << 31)); }
    }
    std::vector<int32_t> ctl(kCtl, 0);
    ctl[C_SEL] = 0;
    ctl[C_NLIVE0] = (int32_t) live.size();
    ctl[C_NEMIT] = (int32_t) (emit.size() / 2);
    {   // the call's small inputs go through pinned host memory and one copy kernel, not the
        // copy engines, which a prefetched encoder copy may keep busy meanwhile
        HostSegments g{};
        size_t need = 0;
        auto plan = [&](void * dst, const void * src, size_t bytes) {
            if (bytes == 0) return;
            g.seg[g.n].src = src;   // host address for now; rebased below
            g.seg[g.n].dst = dst;
            g.seg[g.n].bytes = bytes;
            ++g.n;
            need += (bytes + 15) & ~(size_t) 15;
        };
        if (B > 0) {
            plan(x->ust.p, ust.data(), ust.size() * 4);
            plan(x->frameoff.p, r.frame_off, (size_t) B * 8);
            plan(x->tokregion.p, tokregion.data(), (size_t) B * 8);
            plan(x->bndregion.p, bndregion.data(), (size_t) B * 8);
            plan(x->live.p, live.data(), live.size() * 4);
            plan(x->livef.p, live_frame.data(), live_frame.size() * 8);
            plan(x->emit.p, emit.data(), emit.size() * 4);
            PK_CK(cudaMemsetAsync(x->keys.p, 0, (size_t) B * 32, s));
            PK_CK(cudaMemsetAsync(x->finish.p, 0, (size_t) B * 8, s));
        }
        plan(x->ctl.p, ctl.data(), kCtl * 4);
        if (need > x->pin_cap) {
            if (x->pin) cudaFreeHost(x->pin);
            x->pin = nullptr;
            x->pin_cap = 0;
            PK_CK(cudaHostAlloc(&x->pin, need + need / 4 + 4096, cudaHostAllocMapped));
            x->pin_cap = need + need / 4 + 4096;
        }
        void * pin_dev = nullptr;
        PK_CK(cudaHostGetDevicePointer(&pin_dev, x->pin, 0));
        size_t off = 0;
        for (int i = 0; i < g.n; ++i) {
            std::memcpy(static_cast<unsigned char *>(x->pin) + off, g.seg[i].src, g.seg[i].bytes);
            g.seg[i].src = static_cast<unsigned char *>(pin_dev) + off;
            off += (g.seg[i].bytes + 15) & ~(size_t) 15;
        }
        PK_CK(launch_copy_segments(g, s));
        ++r.launches;
    }
    PK_CK(cudaMemsetAsync(x->bar.p, 0, 32, s));
    if (r.h_in) {
        PK_CK(cudaMemcpyAsync(x->h.p, r.h_in, (size_t) L * H * 4, cudaMemcpyDeviceToDevice, s));
        PK_CK(cudaMemcpyAsync(x->c.p, r.c_in, (size_t) L * H * 4, cudaMemcpyDeviceToDevice, s));
        if (use_tc) {   // staged rows of the resumed state (B == 1: buffer 0, layer l is row l)
            PK_CK(launch_stage_rows(r.h_in, L, H, x->tc_hint ? 1 : 2, x->tc_rbh, x->hst.as<unsigned char>(), s));
            ++r.launches;
        }
    }

    LoopParams P{};
    P.H = H; P.J = J; P.L = L; P.V1 = x->V1; P.Vo = x->Vo; P.Nd = x->Nd; P.blank = x->blank;
    P.eou = x->eou; P.eob = x->eob; P.is_tdt = x->type == PK_MODEL_TDT ? 1 : 0;
    P.max_sym = r.msym; P.B = B; P.n_special = x->n_special;
    P.chunk = x->chunk; P.ldx = x->ldx; P.timeout_ns = x->timeout_ns;
    P.test_stall = x->test_stall;
    x->test_stall = 0;   // one-shot
    if (use_tc) {
        P.tc = 1;
        P.hst = x->hst.as<unsigned char>();
        P.xnew = x->xnew.as<unsigned char>();
        P.hidc = x->hidc.as<unsigned char>();
        P.stationary = x->tc_stationary;
        P.sm_weights = x->tc_sm_weights;
        P.rbh = x->tc_rbh; P.rbj = x->tc_rbj; P.area = x->tc_area; P.mb = x->tc_mb;
        P.rpc_j = x->rpc_j; P.rpc_p = x->rpc_p; P.upc = x->upc; P.h_int = x->tc_hint;
        P.q8 = x->math == PK_MATH_Q8 ? 1 : 0;
        P.tcj = x->tcj; P.tcp = x->tcp;
        for (int l = 0; l < L; ++l) P.tcl[l] = x->tcl[l];
        P.g0 = x->g0.as<float>();
    }
    {
        int64_t tmax = 0;
        for (int b = 0; b < B; ++b) tmax = std::max<int64_t>(tmax, r.n_frames[b]);
        P.max_iters = (int) std::min<int64_t>(tmax * (msym1 + 1) + 2, 1 << 30);
    }
    P.embed = x->embed.as<float>();
    for (int l = 0; l < L; ++l) {
        P.w_ih[l] = x->w_ih[l].as<float>(); P.w_hh[l] = x->w_hh[l].as<float>();
        P.b_ih[l] = x->b_ih[l].as<float>(); P.b_hh[l] = x->b_hh[l].as<float>();
    }
    P.pred_w = x->pred_w.as<float>(); P.pred_b = x->pred_b.as<float>();
    P.out_w = x->out_w.as<float>(); P.out_b = x->out_b.as<float>();
    P.durations = x->durations.as<int32_t>(); P.special = x->special.as<uint8_t>();
    P.encp = x->encp.as<float>(); P.frame_off = x->frameoff.as<int64_t>();
    P.h = x->h.as<float>(); P.c = x->c.as<float>(); P.predp = x->predp.as<float>();
    P.hid = x->hid.as<float>(); P.ust = x->ust.as<int32_t>();
    P.keys = x->keys.as<unsigned long long>(); P.live = x->live.as<int32_t>();
    P.live_frame = x->livef.as<int64_t>();
    P.emit = x->emit.as<int32_t>(); P.ctl = x->ctl.as<int32_t>(); P.bar = x->bar.as<unsigned>();
    P.t_start = x->tstart.as<unsigned long long>(); P.finish_ns = x->finish.as<unsigned long long>();
    P.prof = x->prof.as<unsigned long long>();
    P.tok_out = x->tok.as<int32_t>(); P.tok_region = x->tokregion.as<int64_t>();
    P.bnd_out = x->bnd.as<int32_t>(); P.bnd_region = x->bndregion.as<int64_t>();
    if (r.trace && r.trace->max_steps > 0 && B > 0) {
        const pk_trace & t = *r.trace;
        const size_t S = (size_t) t.max_steps;
        P.trace_steps = t.max_steps;
        PK_CK(x->tr_logits.ensure((size_t) B * S * x->Vo * 4));
        PK_CK(x->tr_h.ensure((size_t) B * S * L * H * 4));
        PK_CK(x->tr_c.ensure((size_t) B * S * L * H * 4));
        PK_CK(x->tr_tok.ensure((size_t) B * S * 4));
        PK_CK(x->tr_dur.ensure((size_t) B * S * 4));
        PK_CK(cudaMemsetAsync(x->tr_logits.p, 0, (size_t) B * S * x->Vo * 4, s));
        PK_CK(cudaMemsetAsync(x->tr_h.p, 0, (size_t) B * S * L * H * 4, s));
        PK_CK(cudaMemsetAsync(x->tr_c.p, 0, (size_t) B * S * L * H * 4, s));
        PK_CK(cudaMemsetAsync(x->tr_tok.p, 0xFF, (size_t) B * S * 4, s));
        PK_CK(cudaMemsetAsync(x->tr_dur.p, 0xFF, (size_t) B * S * 4, s));
        P.tr_logits = x->tr_logits.as<float>(); P.tr_h = x->tr_h.as<float>();
        P.tr_c = x->tr_c.as<float>(); P.tr_tok = x->tr_tok.as<int32_t>();
        P.tr_dur = x->tr_dur.as<int32_t>();
        if (t.forced_token) {
            PK_CK(x->tr_ftok.ensure((size_t) B * S * 4));
            PK_CK(x->tr_fdur.ensure((size_t) B * S * 4));
            PK_CK(cudaMemcpyAsync(x->tr_ftok.p, t.forced_token, (size_t) B * S * 4, cudaMemcpyHostToDevice, s));
            if (t.forced_dur_idx)
                PK_CK(cudaMemcpyAsync(x->tr_fdur.p, t.forced_dur_idx, (size_t) B * S * 4, cudaMemcpyHostToDevice, s));
            else
                PK_CK(cudaMemsetAsync(x->tr_fdur.p, 0, (size_t) B * S * 4, s));
            P.forced_tok = x->tr_ftok.as<int32_t>();
            P.forced_dur = x->tr_fdur.as<int32_t>();
        }
    }
    // Fresh batches that start with many live utterances run their first iterations on
    // the tcgen05 bulk loop; the persistent loop continues where it stops.
    // (every live utterance must start from its init step: the bulk loop's first
    // iteration computes pred-proj for the emit list only)
    bool all_fresh = B > 0;
    for (int b = 0; b < B && all_fresh; ++b)
        all_fresh = r.fresh[b] != 0 || !(r.n_frames[b] > 0 && r.t0[b] < r.n_frames[b]);
    const bool use_bulk = use_tc && x->math == PK_MATH_TC && x->bulk_ok && x->bulk_min_live > 0 && all_fresh &&
                          (int) live.size() >= x->bulk_min_live && B <= x->grid * bulk_threads();
    BulkParams q{};
    if (use_bulk) {
        PK_CK(x->h16.ensure((2 * (size_t) L * Bs + 1) * H * 4));   // + one zero row (reset h_prev)
        PK_CK(x->x16.ensure((size_t) L * Bs * H * 4));
        PK_CK(x->dcount.ensure((size_t) x->grid * 8));
        q.P = P;
        q.min_live = x->bulk_min_live;
        // LSTM and pred-proj as int8 digit planes (kind::i8) when prepared, else f16 halves
        const bool bi8 = x->bulk_i8 && x->bulk.i8_ok;
        for (int l = 0; l < L; ++l) q.gl[l] = bi8 ? x->bulk.gli[l] : x->bulk.gl[l];
        q.gp = bi8 ? x->bulk.gpi : x->bulk.gp;
        q.g0b = bi8 ? x->bulk.g0b : nullptr;
        q.gj = x->bulk.gj;
        q.lbias = x->bulk.lbias;
        q.e16 = x->bulk.e16;
        q.h16 = x->h16.as<unsigned char>();
        q.x16 = x->x16.as<unsigned char>();
        q.dcount = x->dcount.as<int2>();
        // the compact activation rows as TMA boxes (row strides are multiples of 16 bytes)
        q.tma_a = x->bulk_tma_a;
        if (q.tma_a) {
            PK_CK(bulk_row_map(q.map_x16, x->x16.p, (long long) L * Bs, 4LL * H));
            PK_CK(bulk_row_map(q.map_hid, x->hidc.p, (long long) Bs, (long long) x->tc_rbj));
            q.h16_zero_row = (int) (2 * (size_t) L * Bs);
            PK_CK(cudaMemsetAsync(x->h16.as<unsigned char>() + (size_t) q.h16_zero_row * 4 * H, 0, (size_t) 4 * H, s));
            PK_CK(bulk_row_map_gather(q.map_h16, x->h16.p, (long long) q.h16_zero_row + 1, 4LL * H));
        }
        // screened joint (not for trace runs, which report the GEMM's own logits)
        const bool scr = x->bulk_screen_min > 0 && P.trace_steps == 0 && bulk_screen_supported(x->J) &&
                         x->Vo < 0xFFFF && x->V1 >= 64 && x->bulk.wnorm != nullptr;
        q.screen_min = scr ? x->bulk_screen_min : 0;
        if (scr) {
            q.jsum_stride = (x->Vo + 63) / 64;
            q.n_scr = (x->V1 / 64) * 64;
            PK_CK(x->norm2.ensure(Bs * 4));
            PK_CK(x->jsum.ensure(Bs * (size_t) q.jsum_stride * 32));
            PK_CK(cudaMemsetAsync(x->norm2.p, 0, Bs * 4, s));
            q.norm2 = x->norm2.as<float>();
            q.jsum = x->jsum.as<uint4>();
            q.wnorm = x->bulk.wnorm;
        }
        PK_CK(x->bprof.ensure(20 * 8));
        PK_CK(cudaMemsetAsync(x->bprof.p, 0, 20 * 8, s));
        q.prof = x->bprof.as<unsigned long long>();
        P.resume = 1;
    }
    PK_CK(cudaEventRecord(x->ev[3], s));
    if (use_bulk) {
        PK_CK(launch_bulk(q, x->grid, s));
        ++r.launches;
    }
    PK_CK(cudaEventRecord(x->ev[6], s));
    if (B > 0) {
        PK_CK(launch_step_loop(P, x->grid, use_tc ? x->tc_smem : x->smem, s));
        ++r.launches;
    }
    PK_CK(cudaEventRecord(x->ev[4], s));
    r.ust.assign((size_t) B * kUst, 0);
    r.ctl.assign(kCtl, 0);
    if (B > 0) PK_CK(cudaMemcpyAsync(r.ust.data(), x->ust.p, (size_t) B * kUst * 4, cudaMemcpyDeviceToHost, s));
    PK_CK(cudaMemcpyAsync(r.ctl.data(), x->ctl.p, kCtl * 4, cudaMemcpyDeviceToHost, s));
    PK_CK(cudaMemcpyAsync(r.prof, x->prof.p, 8 * 8, cudaMemcpyDeviceToHost, s));
    if (use_bulk) PK_CK(cudaMemcpyAsync(r.bprof, x->bprof.p, 20 * 8, cudaMemcpyDeviceToHost, s));
    PK_CK(cudaStreamSynchronize(s));
    PK_CK(cudaEventElapsedTime(&r.ms_encproj, x->ev[1], x->ev[2]));
    PK_CK(cudaEventElapsedTime(&r.ms_loop, x->ev[3], x->ev[4]));
    PK_CK(cudaEventElapsedTime(&r.ms_bulk, x->ev[3], x->ev[6]));
    if (ep_tc && frames > 0) {
        int ep_err = 0;
        PK_CK(copy_sync(x, &ep_err, x->ep_err.p, sizeof(int), cudaMemcpyDeviceToHost));
        if (ep_err != 0) {
            PK_CK(cudaMemsetAsync(x->ep_err.p, 0, sizeof(int), s));
            return fail(PK_ERR_TIMEOUT, "enc-proj: a pipeline wait exceeded %lld us", x->timeout_ns / 1000);
        }
    }
    if (r.ctl[C_ERR] != 0) {
        const int code = r.ctl[C_ERR];
        if (code == PK_ERR_TIMEOUT)
            return fail(PK_ERR_TIMEOUT, "step loop: a grid-barrier wait exceeded %lld us",
                        x->timeout_ns / 1000);
        return fail((pk_status) code, "step loop: device index check failed (utterance %d)",
                    r.ctl[C_ERRINFO]);
    }
    if (r.trace && r.trace->max_steps > 0 && B > 0) {
        const pk_trace & t = *r.trace;
        const size_t S = (size_t) t.max_steps;
        if (t.logits) PK_CK(copy_sync(x, t.logits, x->tr_logits.p, (size_t) B * S * x->Vo * 4, cudaMemcpyDeviceToHost));
        if (t.h) PK_CK(copy_sync(x, t.h, x->tr_h.p, (size_t) B * S * L * H * 4, cudaMemcpyDeviceToHost));
        if (t.c) PK_CK(copy_sync(x, t.c, x->tr_c.p, (size_t) B * S * L * H * 4, cudaMemcpyDeviceToHost));
        if (t.argmax_token) PK_CK(copy_sync(x, t.argmax_token, x->tr_tok.p, (size_t) B * S * 4, cudaMemcpyDeviceToHost));
        if (t.argmax_dur_idx) PK_CK(copy_sync(x, t.argmax_dur_idx, x->tr_dur.p, (size_t) B * S * 4, cudaMemcpyDeviceToHost));
    }
    return PK_OK;
}

// Compaction of per-utterance regions into the caller's result buffers.
pk_status emit_results(pk_ctx * x, Run & r, pk_result * res) {
    const int B = r.B;
    cudaStream_t s = x->stream;
    PK_CK(x->offsets.ensure((size_t) (B + 1) * 8));
    PK_CK(x->boffsets.ensure((size_t) (B + 1) * 8));
    int64_t ntok = 0, nbnd = 0, nsteps = 0;
    for (int b = 0; b < B; ++b) {
        ntok += r.ust[(size_t) b * kUst + U_NTOK];
        nbnd += r.ust[(size_t) b * kUst + U_NBND];
        nsteps += r.ust[(size_t) b * kUst + U_STEPS];
    }
    res->tokens_needed = ntok;
    res->eou_bounds_needed = nbnd;
    res->total_steps = nsteps;
    res->loop_iterations = r.ctl[C_ITERS];
    res->emit_iterations = r.ctl[C_EMITITERS];
    for (int i = 0; i < 8; ++i) res->phase_ms[i] = (double) r.prof[i] * 1e-6;
    res->encproj_ms = r.ms_encproj;
    res->loop_ms = r.ms_loop;
    res->bulk_ms = r.ms_bulk;
    res->bulk_iterations = r.ctl[C_BULKITERS];
    for (int i = 0; i < 20; ++i) res->bulk_phase_ms[i] = (double) r.bprof[i] * 1e-6;
    res->bulk_steps = r.ctl[C_BULKSTEPS];
    res->bulk_lstm_steps = r.ctl[C_BULKEMITS];
    res->bulk_screened_steps = r.ctl[C_BULKSCREENED];
    if (ntok > res->tokens_cap || (ntok > 0 && !res->tokens))
        return fail(PK_ERR_CAPACITY, "token buffer holds %lld, %lld needed", (long long) res->tokens_cap,
                    (long long) ntok);
    if (res->eou_bounds && nbnd > res->eou_bounds_cap)
        return fail(PK_ERR_CAPACITY, "boundary buffer holds %lld, %lld needed",
                    (long long) res->eou_bounds_cap, (long long) nbnd);
    const bool dev = res->results_on_device != 0;
    if (dev && ((reinterpret_cast<uintptr_t>(res->tokens) | reinterpret_cast<uintptr_t>(res->steps) |
                 reinterpret_cast<uintptr_t>(res->eou_bounds)) & 3u))
        return fail(PK_ERR_INVALID, "device result buffers must be 4-byte aligned");
    PK_CK(launch_scan(x->ust.as<int32_t>(), B, U_NTOK, x->offsets.as<int64_t>(), s));
    ++r.launches;
    if (dev) {
        if (res->tokens && B > 0) {
            PK_CK(launch_gather(x->ust.as<int32_t>(), B, U_NTOK, x->tok.as<int32_t>(),
                                x->tokregion.as<int64_t>(), x->offsets.as<int64_t>(), res->tokens, s));
            ++r.launches;
        }
        if (res->token_offsets)
            PK_CK(cudaMemcpyAsync(res->token_offsets, x->offsets.p, (size_t) (B + 1) * 8, cudaMemcpyDeviceToDevice, s));
        if (res->steps && B > 0) {
            PK_CK(launch_extract_field(x->ust.as<int32_t>(), B, U_STEPS, res->steps, s));
            ++r.launches;
        }
    } else {
        PK_CK(x->compact.ensure((size_t) std::max<int64_t>(ntok, 1) * 4));
        PK_CK(launch_gather(x->ust.as<int32_t>(), B, U_NTOK, x->tok.as<int32_t>(),
                            x->tokregion.as<int64_t>(), x->offsets.as<int64_t>(), x->compact.as<int32_t>(), s));
        if (B > 0) ++r.launches;
        if (ntok > 0) PK_CK(cudaMemcpyAsync(res->tokens, x->compact.p, (size_t) ntok * 4, cudaMemcpyDeviceToHost, s));
        if (res->token_offsets)
            PK_CK(cudaMemcpyAsync(res->token_offsets, x->offsets.p, (size_t) (B + 1) * 8, cudaMemcpyDeviceToHost, s));
        if (res->steps)
            for (int b = 0; b < B; ++b) res->steps[b] = r.ust[(size_t) b * kUst + U_STEPS];
    }
    if (res->eou_bounds && x->type == PK_MODEL_EOU) {
        PK_CK(launch_scan(x->ust.as<int32_t>(), B, U_NBND, x->boffsets.as<int64_t>(), s));
        r.launches += B > 0 ? 2 : 1;
        int32_t * dst = res->eou_bounds;
        if (!dev) {
            PK_CK(x->bcompact.ensure((size_t) std::max<int64_t>(nbnd, 1) * 4));
            dst = x->bcompact.as<int32_t>();
        }
        PK_CK(launch_gather(x->ust.as<int32_t>(), B, U_NBND, x->bnd.as<int32_t>(),
                            x->bndregion.as<int64_t>(), x->boffsets.as<int64_t>(), dst, s));
        if (!dev && nbnd > 0)
            PK_CK(cudaMemcpyAsync(res->eou_bounds, dst, (size_t) nbnd * 4, cudaMemcpyDeviceToHost, s));
        if (res->eou_offsets)
            PK_CK(cudaMemcpyAsync(res->eou_offsets, x->boffsets.p, (size_t) (B + 1) * 8,
                                  dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, s));
    }
    if (res->finish_ms && B > 0) {
        std::vector<unsigned long long> fin((size_t) B);
        unsigned long long t0 = 0;
        PK_CK(cudaMemcpyAsync(fin.data(), x->finish.p, (size_t) B * 8, cudaMemcpyDeviceToHost, s));
        PK_CK(cudaMemcpyAsync(&t0, x->tstart.p, 8, cudaMemcpyDeviceToHost, s));
        PK_CK(cudaStreamSynchronize(s));
        for (int b = 0; b < B; ++b)
            res->finish_ms[b] = fin[(size_t) b] > t0 ? (float) ((double) (fin[(size_t) b] - t0) * 1e-6) : 0.0f;
    }
    PK_CK(cudaEventRecord(x->ev[5], s));
    PK_CK(cudaStreamSynchronize(s));
    float tot = 0.f;
    PK_CK(cudaEventElapsedTime(&tot, x->ev[0], x->ev[5]));
    res->total_ms = tot;
    res->kernel_launches = r.launches;
    return PK_OK;
}

pk_status batch_run(pk_ctx * x, const pk_batch * b, const pk_trace * trace, pk_result * res) {
    if (!x || !b || !res) return fail(PK_ERR_INVALID, "null argument");
    if (b->d_enc != x->De)
        return fail(PK_ERR_DMODEL, "encoder d_model mismatch (%d vs %d)", b->d_enc, x->De);
    if (b->B < 0) return fail(PK_ERR_INVALID, "B < 0");
    if (b->B > 0 && (!b->frame_offsets || !b->n_frames)) return fail(PK_ERR_INVALID, "null offsets");
    if (b->enc_on_device && (reinterpret_cast<uintptr_t>(b->enc) & 3u))
        return fail(PK_ERR_INVALID, "device encoder output must be 4-byte aligned");
    PK_CK(cudaSetDevice(x->device));
    Run r;
    r.enc = b->enc;
    r.enc_dev = b->enc_on_device != 0;
    r.B = b->B;
    r.frame_off = b->frame_offsets;
    r.n_frames = b->n_frames;
    r.msym = b->max_symbols_per_step > 0 ? b->max_symbols_per_step : x->max_sym;
    r.ticket = b->prefetch_ticket;
    r.trace = trace;
    const size_t n = (size_t) std::max(b->B, 0);
    r.t0.assign(n, 0); r.sym0.assign(n, 0); r.nbefore.assign(n, 0); r.segstart.assign(n, 0);
    r.last.assign(n, -1); r.symx.assign(n, 0); r.fresh.assign(n, 0);
    for (int i = 0; i < b->B; ++i)   // tdt_decode_window initialises only when n_frames > 0 (:879-883)
        r.fresh[(size_t) i] = (x->type == PK_MODEL_EOU || b->n_frames[i] > 0) ? 1 : 0;
    PK_TRY(run_loop(x, r));
    return emit_results(x, r, res);
}

}  // namespace

namespace {

// Modelled cost of one step-loop iteration with n live utterances (microseconds,
// TDT-0.6b on one B200 at the default hand-over of 128 live): the persistent loop
// below 128, the bulk loop from 128 up. Piecewise linear; the knot values are a
// least-squares fit to the measured call times of 29 shards of the 4096-utterance
// log-normal batch (1, 2, 4 and 8 shards, two partitions), every one reproduced
// within 4 %. Only the shape matters to the partition, which compares shards.
double iteration_cost(int64_t n) {
    static const double px[] = {1, 16, 32, 64, 127}, py[] = {19.1, 21.7, 34.0, 43.6, 76.8};
    static const double bx[] = {128, 256, 1024, 4096}, by[] = {70.9, 84.5, 141.0, 346.2};
    auto interp = [](const double * x, const double * y, int m, double v) {
        if (v <= x[0]) return y[0];
        for (int i = 1; i < m; ++i)
            if (v <= x[i]) return y[i - 1] + (y[i] - y[i - 1]) * (v - x[i - 1]) / (x[i] - x[i - 1]);
        return y[m - 1] + (y[m - 1] - y[m - 2]) * (v - x[m - 1]) / (x[m - 1] - x[m - 2]);
    };
    if (n <= 0) return 0.0;
    return n < 128 ? interp(px, py, 5, (double) n) : interp(bx, by, 4, (double) n);
}

// Enc-proj per frame in the same units (4.95 ns per frame measured, over ~0.52 decode
// steps per frame, since the partition counts frames as steps).
constexpr double kFrameCost = 0.0095;

}  // namespace

extern "C" {

const char * pk_last_error(void) { return g_err.c_str(); }
int32_t pk_abi_version(void) { return PK_ABI_VERSION; }

pk_status pk_create(const pk_model_desc * d, int device, pk_ctx ** out) {
    if (!out) return fail(PK_ERR_INVALID, "null output pointer");
    *out = nullptr;
    PK_TRY(validate_desc(d));
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0)
        return fail(PK_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= ndev) return fail(PK_ERR_NO_DEVICE, "device %d of %d", device, ndev);
    cudaDeviceProp prop;
    PK_CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10 || prop.minor != 0)
        return fail(PK_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a only",
                    device, prop.major, prop.minor);
    if (!prop.cooperativeLaunch) return fail(PK_ERR_NO_DEVICE, "device lacks cooperative launch");
    PK_CK(cudaSetDevice(device));
    pk_ctx * x = new pk_ctx();
    x->device = device;
    x->sm_count = prop.multiProcessorCount;
    x->type = d->model_type;
    x->H = d->pred_hidden; x->J = d->joint_hidden; x->De = d->d_enc; x->L = d->n_layers;
    x->V = d->vocab_size; x->V1 = d->vocab_size + 1;
    x->Nd = x->type == PK_MODEL_TDT ? d->num_durations : 0;
    x->Vo = x->V1 + x->Nd;
    x->blank = d->blank_id;
    x->max_sym = d->max_symbols_per_step > 0 ? d->max_symbols_per_step : (x->type == PK_MODEL_TDT ? 10 : 5);
    if (x->type == PK_MODEL_EOU) {
        x->eou = d->eou_id >= 0 ? d->eou_id : d->vocab_size - 2;
        x->eob = d->eob_id >= 0 ? d->eob_id : d->vocab_size - 1;
    }
    auto cleanup = [&](pk_status s) { pk_destroy(x); return s; };
    if (cudaStreamCreateWithFlags(&x->stream, cudaStreamNonBlocking) != cudaSuccess)
        return cleanup(fail(PK_ERR_CUDA, "stream creation failed"));
    for (auto & e : x->ev)
        if (cudaEventCreate(&e) != cudaSuccess) return cleanup(fail(PK_ERR_CUDA, "event creation failed"));
    // the copy stream of pk_prefetch_batch (created here so that no prefetch pays for it)
    if (cudaStreamCreateWithFlags(&x->cstream, cudaStreamNonBlocking) != cudaSuccess)
        return cleanup(fail(PK_ERR_CUDA, "stream creation failed"));
    for (auto & e : x->cev)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
            return cleanup(fail(PK_ERR_CUDA, "event creation failed"));
    DevBuf scratch;
    pk_status st = PK_OK;
    auto up = [&](const pk_tensor & t, int64_t keep, DevBuf & dst, const char * name) {
        if (st == PK_OK) st = upload(x, t, keep, dst, scratch, name);
    };
    up(d->embed, x->V1, x->embed, "predict.embed.weight");
    for (int l = 0; l < x->L; ++l) {
        up(d->lstm[l].w_ih, 1 << 30, x->w_ih[l], "lstm.w_ih");
        up(d->lstm[l].w_hh, 1 << 30, x->w_hh[l], "lstm.w_hh");
        up(d->lstm[l].b_ih, 1, x->b_ih[l], "lstm.b_ih");
        up(d->lstm[l].b_hh, 1, x->b_hh[l], "lstm.b_hh");
    }
    up(d->joint_enc_w, 1 << 30, x->enc_w, "joint.enc.weight");
    up(d->joint_enc_b, 1, x->enc_b, "joint.enc.bias");
    up(d->joint_pred_w, 1 << 30, x->pred_w, "joint.pred.weight");
    up(d->joint_pred_b, 1, x->pred_b, "joint.pred.bias");
    up(d->joint_out_w, x->Vo, x->out_w, "joint.out.weight");
    scratch.release();
    if (st != PK_OK) return cleanup(st);
    {   // joint.out.bias: keep the first Vo entries
        pk_tensor ob = d->joint_out_b;
        if (ob.type != PK_GGML_F32 && ob.type != PK_GGML_F16)
            return cleanup(fail(PK_ERR_MODEL, "joint.out.bias must be f32/f16"));
        ob.ne0 = x->Vo;
        ob.ne1 = 1;
        DevBuf sc;
        st = upload(x, ob, 1, x->out_b, sc, "joint.out.bias");
        sc.release();
        if (st != PK_OK) return cleanup(st);
    }
    std::vector<int32_t> durs(d->durations ? d->durations : nullptr,
                              d->durations ? d->durations + x->Nd : nullptr);
    if (durs.empty()) durs.push_back(0);
    if (x->durations.ensure(durs.size() * 4) != cudaSuccess ||
        copy_sync(x, x->durations.p, durs.data(), durs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return cleanup(fail(PK_ERR_CUDA, "durations upload failed"));
    std::vector<uint8_t> special;
    if (x->type == PK_MODEL_EOU && d->special_piece && d->n_vocab_pieces > 0)
        special.assign(d->special_piece, d->special_piece + d->n_vocab_pieces);
    x->n_special = (int) special.size();
    if (special.empty()) special.push_back(0);
    if (x->special.ensure(special.size()) != cudaSuccess ||
        copy_sync(x, x->special.p, special.data(), special.size(), cudaMemcpyHostToDevice) != cudaSuccess)
        return cleanup(fail(PK_ERR_CUDA, "special-piece table upload failed"));

    // Step-loop launch shape: one CTA per SM, activation chunks sized to shared memory.
    x->grid = x->sm_count;
    x->ldx = ((std::max(2 * x->H, x->J) + 3) / 4) * 4;
    x->chunk = 32;
    const size_t smem_cap = std::min<size_t>(prop.sharedMemPerBlockOptin - step_loop_static_smem(0), 200 * 1024);
    while (x->chunk > 1 && step_loop_smem_bytes(x->chunk, x->ldx, x->H, x->grid) > smem_cap) x->chunk >>= 1;
    x->smem = step_loop_smem_bytes(x->chunk, x->ldx, x->H, x->grid);
    if (x->smem > smem_cap) return cleanup(fail(PK_ERR_MODEL, "hidden sizes too large for shared memory"));
    if (step_loop_configure(x->smem, 0) != cudaSuccess)
        return cleanup(fail(PK_ERR_CUDA, "cannot configure %zu B of shared memory", x->smem));
    int per_sm = 0;
    if (step_loop_occupancy(x->smem, 0, &per_sm) != cudaSuccess || per_sm < 1)
        return cleanup(fail(PK_ERR_CUDA, "step loop does not fit one CTA per SM"));
    // dynamic shared memory may use what the kernel's static arrays leave
    st = setup_tc(x, d, (size_t) prop.sharedMemPerBlockOptin - step_loop_static_smem(1));
    if (st != PK_OK) return cleanup(st);
    setup_encproj(x, (size_t) prop.sharedMemPerBlockOptin);
    x->math = x->tc_ok ? PK_MATH_TC : PK_MATH_F32;
    // the tcgen05 loop for iterations with many live utterances (tensor-core models only)
    if (x->tc_ok && bulk_supported(x->H, x->J, x->L) && bulk_smem_bytes() <= (size_t) prop.sharedMemPerBlockOptin) {
        int bps = 0;
        if (bulk_configure() == cudaSuccess && bulk_occupancy(&bps) == cudaSuccess && bps >= 1) {
            const float * wih[kMaxLayers], * whh[kMaxLayers], * bih[kMaxLayers], * bhh[kMaxLayers];
            for (int l = 0; l < x->L; ++l) {
                wih[l] = x->w_ih[l].as<float>(); whh[l] = x->w_hh[l].as<float>();
                bih[l] = x->b_ih[l].as<float>(); bhh[l] = x->b_hh[l].as<float>();
            }
            // matrices whose source tensors are all f16 have zero lo halves
            int f16w[kMaxLayers + 2] = {};
            for (int l = 0; l < x->L; ++l)
                f16w[l] = d->lstm[l].w_ih.type == PK_GGML_F16 && d->lstm[l].w_hh.type == PK_GGML_F16;
            f16w[x->L] = d->joint_pred_w.type == PK_GGML_F16;
            f16w[x->L + 1] = d->joint_out_w.type == PK_GGML_F16;
            if (bulk_prepare(x->bulk, x->H, x->J, x->L, x->Vo, x->V1, x->embed.as<float>(), wih, whh, bih, bhh,
                             x->pred_w.as<float>(), x->out_w.as<float>(), f16w, x->g0.as<float>(),
                             x->stream) != cudaSuccess) {
                bulk_release(x->bulk);
                return cleanup(fail(PK_ERR_CUDA, "bulk-loop weight preparation failed"));
            }
            x->bulk_ok = 1;
            x->weight_bytes += x->bulk.bytes;
        }
    }
    // pk_decode_noalloc allocates nothing: its module (and static scratch array) is
    // loaded now, and one 1-frame decode on the f32 loop it runs sizes the context's
    // local memory for that kernel here rather than at its first call
    if (noalloc_prepare(device) != PK_OK) return cleanup(fail(PK_ERR_CUDA, "no-allocation path set-up failed"));
    {
        const int math = x->math;
        x->math = PK_MATH_F32;
        std::vector<float> frame((size_t) x->De, 0.0f);
        const int64_t off0 = 0;
        const int32_t one = 1;
        pk_batch wb{};
        wb.enc = frame.data();
        wb.B = 1;
        wb.d_enc = x->De;
        wb.frame_offsets = &off0;
        wb.n_frames = &one;
        int32_t tok[64];
        int64_t toff[2];
        pk_result wr{};
        wr.tokens = tok;
        wr.tokens_cap = 64;
        wr.token_offsets = toff;
        const pk_status ws = batch_run(x, &wb, nullptr, &wr);
        x->math = math;
        if (ws != PK_OK) return cleanup(ws);
    }
    *out = x;
    return PK_OK;
}

void pk_destroy(pk_ctx * x) {
    if (!x) return;
    cudaSetDevice(x->device);
    if (x->stream) cudaStreamSynchronize(x->stream);
    if (x->cstream) cudaStreamSynchronize(x->cstream);
    for (DevBuf * b : x->all_bufs()) b->release();
    bulk_release(x->bulk);
    if (x->pin) cudaFreeHost(x->pin);
    for (auto & e : x->ev)
        if (e) cudaEventDestroy(e);
    for (auto & e : x->cev)
        if (e) cudaEventDestroy(e);
    if (x->stream) cudaStreamDestroy(x->stream);
    if (x->cstream) cudaStreamDestroy(x->cstream);
    delete x;
}

pk_status pk_get_info(const pk_ctx * x, pk_info * i) {
    if (!x || !i) return fail(PK_ERR_INVALID, "null argument");
    i->model_type = x->type; i->d_enc = x->De; i->pred_hidden = x->H; i->joint_hidden = x->J;
    i->n_layers = x->L; i->vocab_size = x->V; i->blank_id = x->blank; i->num_durations = x->Nd;
    i->v_plus_1 = x->V1; i->v_out = x->Vo; i->eou_id = x->eou; i->eob_id = x->eob;
    i->max_symbols_per_step = x->max_sym; i->device = x->device; i->sm_count = x->sm_count;
    i->grid_ctas = x->grid; i->weight_bytes_device = x->weight_bytes;
    return PK_OK;
}

pk_status pk_set_option(pk_ctx * x, int32_t opt, int64_t v) {
    if (!x) return fail(PK_ERR_INVALID, "null context");
    switch (opt) {
        case PK_OPT_TIMEOUT_US:
            if (v <= 0) return fail(PK_ERR_INVALID, "timeout must be > 0");
            x->timeout_ns = v * 1000;
            return PK_OK;
        case PK_OPT_MATH:
            if (v == PK_MATH_TC && !x->tc_ok)
                return fail(PK_ERR_INVALID, "tensor-core math needs q8_0/f16 step-loop weights and H, J multiples of 32");
            if (v == PK_MATH_Q8 && !(x->tc_ok && x->tc_hint && x->tcj.is_i8))
                return fail(PK_ERR_INVALID, "q8_0-activation math needs q8_0 weights in every step-loop matrix");
            if (v != PK_MATH_F32 && v != PK_MATH_TC && v != PK_MATH_Q8)
                return fail(PK_ERR_INVALID, "unsupported math mode %lld", (long long) v);
            x->math = (int) v;
            return PK_OK;
        case PK_OPT_MAX_SYMBOLS:
            if (v <= 0) return fail(PK_ERR_INVALID, "max_symbols must be > 0");
            x->max_sym = (int) v;
            return PK_OK;
        case PK_OPT_TEST_STALL:
            x->test_stall = v != 0 ? 1 : 0;
            return PK_OK;
        case PK_OPT_BULK_MIN_LIVE:
            if (v < 0) return fail(PK_ERR_INVALID, "bulk threshold must be >= 0");
            x->bulk_min_live = (int) std::min<int64_t>(v, 1 << 30);
            return PK_OK;
        case PK_OPT_BULK_TMA_A:
            x->bulk_tma_a = v != 0 ? 1 : 0;
            return PK_OK;
        case PK_OPT_BULK_I8:
            x->bulk_i8 = v != 0 ? 1 : 0;
            return PK_OK;
        case PK_OPT_BULK_SCREEN:
            if (v < 0) return fail(PK_ERR_INVALID, "screening threshold must be >= 0");
            x->bulk_screen_min = (int) std::min<int64_t>(v, 1 << 30);
            return PK_OK;
        default:
            return fail(PK_ERR_INVALID, "unknown option %d", opt);
    }
}

int64_t pk_tokens_capacity(const int32_t * n_frames, int32_t B, int32_t msym) {
    int64_t s = 0;
    const int m = msym > 0 ? msym : 1;
    for (int b = 0; n_frames && b < B; ++b) s += (int64_t) std::max(n_frames[b], 0) * m;
    return s;
}

pk_status pk_decode_batch(pk_ctx * x, const pk_batch * b, pk_result * res) {
    return batch_run(x, b, nullptr, res);
}

pk_status pk_prefetch_batch(pk_ctx * x, const pk_batch * b, uint64_t * ticket) {
    if (ticket) *ticket = 0;
    if (!x || !b || !ticket) return fail(PK_ERR_INVALID, "null argument");
    if (b->enc_on_device) return fail(PK_ERR_INVALID, "prefetch takes host encoder outputs");
    if (b->d_enc != x->De)
        return fail(PK_ERR_DMODEL, "encoder d_model mismatch (%d vs %d)", b->d_enc, x->De);
    if (b->B < 0) return fail(PK_ERR_INVALID, "B < 0");
    if (b->B > 0 && (!b->frame_offsets || !b->n_frames)) return fail(PK_ERR_INVALID, "null offsets");
    int64_t frames = 0;
    for (int i = 0; i < b->B; ++i) {
        if (b->n_frames[i] < 0) return fail(PK_ERR_INVALID, "n_frames[%d] < 0", i);
        if (b->n_frames[i] > 0) {
            if (b->frame_offsets[i] < 0) return fail(PK_ERR_INVALID, "frame_offsets[%d] < 0", i);
            frames = std::max<int64_t>(frames, b->frame_offsets[i] + b->n_frames[i]);
        }
    }
    if (frames == 0) return PK_OK;            // nothing to copy: ticket 0, the decode copies nothing
    if (!b->enc) return fail(PK_ERR_INVALID, "null encoder output");
    PK_CK(cudaSetDevice(x->device));
    // copy n reuses copy n-2's event: wait for that copy (so its host buffer and,
    // if it was never used, its slot are free), which also bounds the copies in flight.
    // The compute stream is idle between calls (every call synchronises it); waiting
    // for it covers work a failed call left behind that may still read a slot.
    const uint64_t n = x->n_copies;
    PK_CK(cudaEventSynchronize(x->cev[n & 1]));
    PK_CK(cudaStreamSynchronize(x->stream));
    const int q = !x->stg_seq[0] ? 0 : !x->stg_seq[1] ? 1 : (x->stg_seq[0] < x->stg_seq[1] ? 0 : 1);
    x->stg_seq[q] = 0;
    const size_t bytes = (size_t) frames * x->De * 4;
    if (x->stg[q].cap < bytes) {
        PK_CK(cudaStreamSynchronize(x->cstream));   // the other slot's copy may still read into its buffer
        PK_CK(x->stg[q].ensure(bytes));
    }
    PK_CK(cudaMemcpyAsync(x->stg[q].p, b->enc, bytes, cudaMemcpyHostToDevice, x->cstream));
    PK_CK(cudaEventRecord(x->cev[n & 1], x->cstream));
    x->n_copies = n + 1;
    x->stg_frames[q] = frames;
    x->stg_seq[q] = n + 1;
    *ticket = n + 1;
    return PK_OK;
}

pk_status pk_decode_trace(pk_ctx * x, const pk_batch * b, pk_trace * t, pk_result * res) {
    if (!t || t->max_steps < 0) return fail(PK_ERR_INVALID, "bad trace");
    return batch_run(x, b, t, res);
}

pk_status pk_stream_create(pk_ctx * x, pk_stream ** out) {
    if (!x || !out) return fail(PK_ERR_INVALID, "null argument");
    *out = nullptr;
    PK_CK(cudaSetDevice(x->device));
    pk_stream * s = new pk_stream();
    s->ctx = x;
    const size_t n = (size_t) x->L * x->H * 4;
    if (s->h.ensure(n) != cudaSuccess || s->c.ensure(n) != cudaSuccess ||
        cudaMemsetAsync(s->h.p, 0, n, x->stream) != cudaSuccess ||
        cudaMemsetAsync(s->c.p, 0, n, x->stream) != cudaSuccess ||
        cudaStreamSynchronize(x->stream) != cudaSuccess) {
        pk_stream_destroy(s);
        return fail(PK_ERR_OOM, "stream state allocation failed");
    }
    *out = s;
    return PK_OK;
}

void pk_stream_destroy(pk_stream * s) {
    if (!s) return;
    if (s->ctx) cudaSetDevice(s->ctx->device);
    s->h.release();
    s->c.release();
    delete s;
}

namespace {
pk_status stream_run(pk_stream * s, const float * enc, bool enc_dev, int n_frames, int msym,
                     int n_before, bool force_init, Run & r) {
    pk_ctx * x = s->ctx;
    if (enc_dev && (reinterpret_cast<uintptr_t>(enc) & 3u))
        return fail(PK_ERR_INVALID, "device encoder output must be 4-byte aligned");
    const bool fresh = force_init || !s->initialized;
    if (fresh) { s->sym = 0; s->carry = 0; s->last = -1; s->segstart = 0; s->symx = 0; }
    int t0 = 0;
    if (x->type == PK_MODEL_TDT && s->carry > 0 && n_frames > 0) {   // :907-910
        t0 = std::min(s->carry, n_frames);
        s->carry -= t0;
    }
    static const int64_t zero_off = 0;
    r.enc = enc; r.enc_dev = enc_dev; r.B = 1; r.frame_off = &zero_off;
    r.n_frames = &n_frames;
    r.msym = msym;
    r.t0 = {t0}; r.sym0 = {x->type == PK_MODEL_TDT ? s->sym : 0}; r.nbefore = {n_before};
    r.segstart = {s->segstart}; r.last = {s->last}; r.symx = {s->symx}; r.fresh = {fresh ? 1 : 0};
    if (!fresh) { r.h_in = s->h.as<float>(); r.c_in = s->c.as<float>(); }
    PK_TRY(run_loop(x, r));
    const int32_t * u = r.ust.data();
    const size_t LH = (size_t) x->L * x->H;
    PK_CK(cudaMemcpyAsync(s->h.p, x->h.as<float>() + (size_t) u[U_HBUF] * LH, LH * 4,
                          cudaMemcpyDeviceToDevice, x->stream));
    PK_CK(cudaMemcpyAsync(s->c.p, x->c.p, LH * 4, cudaMemcpyDeviceToDevice, x->stream));
    PK_CK(cudaStreamSynchronize(x->stream));
    if (x->type == PK_MODEL_TDT) {
        s->sym = u[U_SYM];
        if (n_frames > 0) s->carry = std::max(0, u[U_T] - n_frames);   // :979
    } else {
        s->symx = u[U_SYMX];
        s->sym = u[U_SYMX];
        s->last = u[U_LAST];
        s->segstart = u[U_SEGSTART];
    }
    s->initialized = 1;
    return PK_OK;
}
}  // namespace

pk_status pk_stream_reset(pk_stream * s) {
    if (!s || !s->ctx) return fail(PK_ERR_INVALID, "null stream");
    PK_CK(cudaSetDevice(s->ctx->device));
    Run r;
    return stream_run(s, nullptr, false, 0, s->ctx->max_sym, 0, true, r);
}

pk_status pk_stream_window(pk_stream * s, const float * enc, int32_t enc_on_device, int32_t n_frames,
                           int32_t d_enc, int32_t msym_in, int32_t n_before, int32_t * tokens,
                           int32_t tokens_cap, int32_t * n_tokens, int32_t * steps,
                           int32_t * bounds, int32_t bounds_cap, int32_t * n_bounds) {
    if (!s || !s->ctx) return fail(PK_ERR_INVALID, "null stream");
    pk_ctx * x = s->ctx;
    if (n_tokens) *n_tokens = 0;
    if (steps) *steps = 0;
    if (n_bounds) *n_bounds = 0;
    if (d_enc != x->De)
        return fail(PK_ERR_DMODEL, "encoder d_model mismatch (%d vs %d)", d_enc, x->De);
    if (x->type == PK_MODEL_TDT && n_frames <= 0) return PK_OK;      // :879
    if (n_frames < 0) n_frames = 0;
    if (n_frames > 0 && !enc) return fail(PK_ERR_INVALID, "null encoder output");
    PK_CK(cudaSetDevice(x->device));
    const int msym = msym_in > 0 ? msym_in : x->max_sym;
    Run r;
    PK_TRY(stream_run(s, enc, enc_on_device != 0, n_frames, msym, n_before, false, r));
    const int32_t * u = r.ust.data();
    const int nt = u[U_NTOK], nb = u[U_NBND];
    if (nt > tokens_cap || (nt > 0 && !tokens))
        return fail(PK_ERR_CAPACITY, "token buffer holds %d, %d needed", tokens_cap, nt);
    if (nt > 0) PK_CK(copy_sync(x, tokens, x->tok.p, (size_t) nt * 4, cudaMemcpyDeviceToHost));
    if (bounds && nb > 0) {
        if (nb > bounds_cap) return fail(PK_ERR_CAPACITY, "boundary buffer holds %d, %d needed", bounds_cap, nb);
        PK_CK(copy_sync(x, bounds, x->bnd.p, (size_t) nb * 4, cudaMemcpyDeviceToHost));
    }
    if (n_tokens) *n_tokens = nt;
    if (steps) *steps = u[U_STEPS];
    if (n_bounds) *n_bounds = nb;
    return PK_OK;
}

pk_status pk_stream_get_state(const pk_stream * s, pk_stream_state * st) {
    if (!s || !s->ctx || !st) return fail(PK_ERR_INVALID, "null argument");
    pk_ctx * x = s->ctx;
    PK_CK(cudaSetDevice(x->device));
    const size_t LH = (size_t) x->L * x->H;
    std::vector<float> h(LH), c(LH);
    PK_CK(copy_sync(x, h.data(), s->h.p, LH * 4, cudaMemcpyDeviceToHost));
    PK_CK(copy_sync(x, c.data(), s->c.p, LH * 4, cudaMemcpyDeviceToHost));
    if (st->h) std::memcpy(st->h, h.data(), LH * 4);
    if (st->c) std::memcpy(st->c, c.data(), LH * 4);
    if (st->pred_out) std::memcpy(st->pred_out, h.data() + (size_t) (x->L - 1) * x->H, (size_t) x->H * 4);
    st->symbols_this_step = s->sym;
    st->carry_frames = s->carry;
    st->initialized = s->initialized;
    st->last_token = s->last;
    st->segment_start_token = s->segstart;
    return PK_OK;
}

pk_status pk_stream_set_state(pk_stream * s, const pk_stream_state * st) {
    if (!s || !s->ctx || !st || !st->h || !st->c) return fail(PK_ERR_INVALID, "null argument");
    pk_ctx * x = s->ctx;
    PK_CK(cudaSetDevice(x->device));
    const size_t LH = (size_t) x->L * x->H;
    PK_CK(copy_sync(x, s->h.p, st->h, LH * 4, cudaMemcpyHostToDevice));
    PK_CK(copy_sync(x, s->c.p, st->c, LH * 4, cudaMemcpyHostToDevice));
    s->sym = st->symbols_this_step;
    s->symx = st->symbols_this_step;
    s->carry = st->carry_frames;
    s->initialized = st->initialized;
    s->last = st->last_token;
    s->segstart = st->segment_start_token;
    return PK_OK;
}

pk_status pk_shard_lpt(const int32_t * n_frames, int32_t B, int32_t n_shards, int32_t * shard_of) {
    if (B < 0 || n_shards <= 0 || (B > 0 && (!n_frames || !shard_of)))
        return fail(PK_ERR_INVALID, "bad sharding arguments");
    std::vector<int> idx((size_t) B);
    std::iota(idx.begin(), idx.end(), 0);
    std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return n_frames[a] > n_frames[b]; });
    std::vector<int64_t> load((size_t) n_shards, 0);
    for (int i : idx) {
        int best = 0;
        for (int k = 1; k < n_shards; ++k)
            if (load[(size_t) k] < load[(size_t) best]) best = k;
        shard_of[i] = best;
        load[(size_t) best] += std::max(n_frames[i], 0);
    }
    return PK_OK;
}

pk_status pk_shard_balanced(const int32_t * n_frames, int32_t B, int32_t n_shards, int32_t * shard_of) {
    if (B < 0 || n_shards <= 0 || (B > 0 && (!n_frames || !shard_of)))
        return fail(PK_ERR_INVALID, "bad sharding arguments");
    // A shard's call lasts sum_i cost(live_i) over its loop iterations, live_i = its
    // utterances with more than i decode steps; steps are taken proportional to
    // frames. Utterances are placed in descending length, so every member already on
    // a shard is at least as long as the next one: adding t frames to a shard of n
    // adds t * (cost(n + 1) - cost(n)), plus its enc-proj. First fit decreasing against a bound M on
    // every shard's modelled time (each utterance to the lowest shard that stays
    // within M), with M bisected down to the smallest bound that places every
    // utterance: long utterances share shards, whose per-iteration cost barely
    // grows with a few more live, instead of each setting its own shard's time.
    std::vector<int> idx((size_t) B);
    std::iota(idx.begin(), idx.end(), 0);
    std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return n_frames[a] > n_frames[b]; });
    std::vector<double> time((size_t) n_shards);
    std::vector<int64_t> count((size_t) n_shards);
    std::vector<int32_t> trial((size_t) std::max(B, 1));
    auto place = [&](double M) -> bool {
        std::fill(time.begin(), time.end(), 0.0);
        std::fill(count.begin(), count.end(), 0);
        for (int i : idx) {
            const double t = (double) std::max(n_frames[i], 0);
            int k = 0;
            for (; k < n_shards; ++k) {
                const int64_t n = count[(size_t) k];
                const double after = time[(size_t) k] + t * (iteration_cost(n + 1) - iteration_cost(n)) + kFrameCost * t;
                if (after <= M) {
                    time[(size_t) k] = after;
                    ++count[(size_t) k];
                    trial[(size_t) i] = k;
                    break;
                }
            }
            if (k == n_shards) return false;
        }
        return true;
    };
    if (B == 0) return PK_OK;
    // bounds: the longest utterance alone; everything on one shard
    double lo = (double) std::max(n_frames[idx[0]], 0) * (iteration_cost(1) + kFrameCost), hi = 0.0;
    for (size_t r = 0; r < idx.size(); ++r)
        hi += (double) std::max(n_frames[idx[r]], 0) *
              (iteration_cost((int64_t) r + 1) - iteration_cost((int64_t) r) + kFrameCost);
    place(hi);
    std::copy(trial.begin(), trial.begin() + B, shard_of);
    for (int it = 0; it < 64 && hi - lo > 1e-9 * hi; ++it) {
        const double mid = 0.5 * (lo + hi);
        if (place(mid)) {
            hi = mid;
            std::copy(trial.begin(), trial.begin() + B, shard_of);
        } else {
            lo = mid;
        }
    }
    return PK_OK;
}

}  // extern "C"

namespace pk {

pk_status set_error(pk_status s, const char * msg) { return fail(s, "%s", msg); }

void ctx_view(const pk_ctx * x, CtxView * v) {
    v->device = x->device; v->grid = x->grid; v->chunk = x->chunk; v->ldx = x->ldx;
    v->smem = x->smem; v->stream = x->stream;
    v->H = x->H; v->J = x->J; v->De = x->De; v->L = x->L; v->V1 = x->V1; v->Vo = x->Vo;
    v->Nd = x->Nd; v->blank = x->blank; v->eou = x->eou; v->eob = x->eob;
    v->is_tdt = x->type == PK_MODEL_TDT ? 1 : 0; v->max_sym = x->max_sym;
    v->n_special = x->n_special; v->timeout_ns = x->timeout_ns;
    v->embed = x->embed.as<float>();
    for (int l = 0; l < kMaxLayers; ++l) {
        v->w_ih[l] = x->w_ih[l].as<float>(); v->w_hh[l] = x->w_hh[l].as<float>();
        v->b_ih[l] = x->b_ih[l].as<float>(); v->b_hh[l] = x->b_hh[l].as<float>();
    }
    v->enc_w = x->enc_w.as<float>(); v->enc_b = x->enc_b.as<float>();
    v->pred_w = x->pred_w.as<float>(); v->pred_b = x->pred_b.as<float>();
    v->out_w = x->out_w.as<float>(); v->out_b = x->out_b.as<float>();
    v->durations = x->durations.as<int32_t>(); v->special = x->special.as<uint8_t>();
}

}  // namespace pk
