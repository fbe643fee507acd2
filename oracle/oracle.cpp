// oracle.cpp -- TEST INFRASTRUCTURE ONLY: CPU restatement of parakeet.cpp's
// f32 host decoder, used as the parity checker and the timed CPU baseline.
// Never linked into libparakeet_cuda.
//
// Each function cites the reference lines it restates. Compile with
// -O3 -ffast-math -funroll-loops and no -march, the flags of the reference
// library (CMakeLists.txt:327-335).

#include "oracle.h"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace {

// ---- dequantisation (ggml to_float, called at src/parakeet_tdt.cpp:78-95) ----
//
// Restated from the public GGUF block formats, not from ggml's source:
//   F16 : IEEE-754 binary16 per element;
//   Q8_0: blocks of 32 weights {binary16 d; int8 qs[32]}, value = f32(d) * qs[i].
// Both are exact in f32.

float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            int e = -1;
            do { ++e; man <<= 1; } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            bits = sign | ((uint32_t) (127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

bool dequantize(const pk_tensor & t, std::vector<float> & out, std::string & err) {
    if (!t.data) { err = "missing tensor"; return false; }
    const int64_t n = t.ne0 * (t.ne1 > 0 ? t.ne1 : 1);
    out.resize((size_t) n);
    const uint8_t * p = static_cast<const uint8_t *>(t.data);
    if (t.type == PK_GGML_F32) {
        if (t.nbytes < (uint64_t) n * 4) { err = "f32 tensor too small"; return false; }
        std::memcpy(out.data(), p, (size_t) n * 4);
        return true;
    }
    if (t.type == PK_GGML_F16) {
        if (t.nbytes < (uint64_t) n * 2) { err = "f16 tensor too small"; return false; }
        for (int64_t i = 0; i < n; ++i) {
            uint16_t h;
            std::memcpy(&h, p + 2 * i, 2);
            out[(size_t) i] = half_to_float(h);
        }
        return true;
    }
    if (t.type == PK_GGML_Q8_0) {
        if (t.ne0 % 32 != 0) { err = "q8_0 row not a multiple of 32"; return false; }
        const int64_t nb = n / 32;
        if (t.nbytes < (uint64_t) nb * 34) { err = "q8_0 tensor too small"; return false; }
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t * blk = p + b * 34;
            uint16_t dh;
            std::memcpy(&dh, blk, 2);
            const float d = half_to_float(dh);
            const int8_t * qs = reinterpret_cast<const int8_t *>(blk + 2);
            for (int j = 0; j < 32; ++j) out[(size_t) (b * 32 + j)] = (float) qs[j] * d;
        }
        return true;
    }
    err = "unsupported ggml type " + std::to_string(t.type);
    return false;
}

// ---- numerics restated from src/parakeet_tdt.cpp:25-68 ---------------------

int argmax_f32(const float * data, int n) {              // :25-32 (strict >, first index wins)
    int best = 0;
    float best_val = data[0];
    for (int i = 1; i < n; ++i) {
        if (data[i] > best_val) { best_val = data[i]; best = i; }
    }
    return best;
}

float top2_margin(const float * data, int n) {
    if (n < 2) return INFINITY;
    float a = -INFINITY, b = -INFINITY;
    for (int i = 0; i < n; ++i) {
        const float v = data[i];
        if (v > a) { b = a; a = v; } else if (v > b) { b = v; }
    }
    return a - b;
}

inline float sigmoidf_ref(float x) { return 1.0f / (1.0f + std::exp(-x)); }   // :34

void gemv_f32(const float * __restrict W, const float * __restrict x,         // :47-57
              const float * __restrict b, float * __restrict y,
              int out_dim, int in_dim) {
    for (int i = 0; i < out_dim; ++i) {
        const float * __restrict row = W + (size_t) i * in_dim;
        float acc = b ? b[i] : 0.0f;
        #pragma GCC ivdep
        for (int j = 0; j < in_dim; ++j) acc += row[j] * x[j];
        y[i] = acc;
    }
}

void gemv_add_f32(const float * __restrict W, const float * __restrict x,     // :59-68
                  float * __restrict y, int out_dim, int in_dim) {
    for (int i = 0; i < out_dim; ++i) {
        const float * __restrict row = W + (size_t) i * in_dim;
        float acc = 0.0f;
        #pragma GCC ivdep
        for (int j = 0; j < in_dim; ++j) acc += row[j] * x[j];
        y[i] += acc;
    }
}

struct Layer { std::vector<float> w_ih, w_hh, b_ih, b_hh; };

}  // namespace

struct orc_model {
    int type = PK_MODEL_TDT;
    int H = 640, J = 640, De = 1024, L = 2, V1 = 8193, Vo = 8198, Nd = 5;
    int blank = 8192, eou = -1, eob = -1, max_sym = 10;
    std::vector<int32_t> durations;
    std::vector<uint8_t> special;   // EOU <...> pieces
    std::vector<float> embed;
    std::vector<Layer> lstm;
    std::vector<float> enc_w, enc_b, pred_w, pred_b, out_w, out_b;
};

namespace {

struct Scratch {
    std::vector<float> g, layer_in, hidden, tmp, logits;
};

// host_lstm_step, src/parakeet_tdt.cpp:106-142 (identical in parakeet_eou.cpp:78-116)
void lstm_step(const orc_model & W, const float * __restrict x_input,
               float * __restrict h_state, float * __restrict c_state, Scratch & s) {
    const int H = W.H, L = W.L, G = 4 * H;
    s.g.resize((size_t) G);
    s.layer_in.resize((size_t) H);
    const float * x = x_input;
    for (int layer = 0; layer < L; ++layer) {
        const Layer & w = W.lstm[(size_t) layer];
        const float * h_l = h_state + (size_t) layer * H;
        float * c_l = c_state + (size_t) layer * H;
        gemv_f32(w.w_ih.data(), x, w.b_ih.data(), s.g.data(), G, H);
        for (int i = 0; i < G; ++i) s.g[(size_t) i] += w.b_hh[(size_t) i];
        gemv_add_f32(w.w_hh.data(), h_l, s.g.data(), G, H);
        float * h_new = h_state + (size_t) layer * H;
        for (int i = 0; i < H; ++i) {
            const float i_g = sigmoidf_ref(s.g[(size_t) (0 * H + i)]);
            const float f_g = sigmoidf_ref(s.g[(size_t) (1 * H + i)]);
            const float g_g = std::tanh(s.g[(size_t) (2 * H + i)]);
            const float o_g = sigmoidf_ref(s.g[(size_t) (3 * H + i)]);
            const float c_new = f_g * c_l[i] + i_g * g_g;
            c_l[i] = c_new;
            h_new[i] = o_g * std::tanh(c_new);
        }
        std::memcpy(s.layer_in.data(), h_new, (size_t) H * sizeof(float));
        x = s.layer_in.data();
    }
}

// host_joint_step, src/parakeet_tdt.cpp:154-177 (EOU joint_step parakeet_eou.cpp:123-143
// is the same with n_out = V+1)
void joint_step(const orc_model & W, const float * __restrict enc_frame,
                const float * __restrict pred, int n_out, Scratch & s) {
    const int J = W.J, H = W.H, De = W.De;
    s.hidden.resize((size_t) J);
    s.tmp.resize((size_t) J);
    gemv_f32(W.enc_w.data(), enc_frame, W.enc_b.data(), s.hidden.data(), J, De);
    gemv_f32(W.pred_w.data(), pred, W.pred_b.data(), s.tmp.data(), J, H);
    for (int i = 0; i < J; ++i) s.hidden[(size_t) i] += s.tmp[(size_t) i];
    for (int i = 0; i < J; ++i) s.hidden[(size_t) i] = std::max(0.0f, s.hidden[(size_t) i]);
    s.logits.resize((size_t) n_out);
    gemv_f32(W.out_w.data(), s.hidden.data(), W.out_b.data(), s.logits.data(), n_out, J);
}

void copy_pred(const orc_model & W, orc_state * st) {
    std::memcpy(st->pred, st->h + (size_t) (W.L - 1) * W.H, (size_t) W.H * sizeof(float));
}

void trace_state(const orc_model & W, const orc_state * st, orc_trace * tr, int s) {
    if (!tr || s >= tr->max_steps) return;
    const size_t n = (size_t) W.L * W.H;
    if (tr->h) std::memcpy(tr->h + (size_t) s * n, st->h, n * sizeof(float));
    if (tr->c) std::memcpy(tr->c + (size_t) s * n, st->c, n * sizeof(float));
}

bool check(bool ok, const char * what, char * err, int errlen) {
    if (!ok && err && errlen > 0) std::snprintf(err, (size_t) errlen, "%s", what);
    return ok;
}

bool shape_ok(const pk_tensor & t, int64_t ne0, int64_t ne1) {
    return t.data && t.ne0 == ne0 && (ne1 <= 1 ? (t.ne1 <= 1) : t.ne1 == ne1);
}

}  // namespace

extern "C" {

int32_t orc_dequantize(const pk_tensor * t, float * out) {
    if (!t || !out) return 2;
    std::vector<float> v;
    std::string err;
    if (!dequantize(*t, v, err)) return 3;
    std::memcpy(out, v.data(), v.size() * sizeof(float));
    return 0;
}

orc_model * orc_create(const pk_model_desc * d, char * err, int32_t errlen) {
    if (!check(d != nullptr, "null descriptor", err, errlen)) return nullptr;
    orc_model * m = new orc_model();
    orc_model & W = *m;
    W.type = d->model_type;
    W.H = d->pred_hidden; W.J = d->joint_hidden; W.De = d->d_enc; W.L = d->n_layers;
    W.V1 = d->vocab_size + 1;                                   // parakeet_tdt.cpp:593
    W.Nd = (W.type == PK_MODEL_TDT) ? d->num_durations : 0;
    W.Vo = W.V1 + W.Nd;                                         // parakeet_tdt.cpp:594
    W.blank = d->blank_id;
    W.max_sym = d->max_symbols_per_step > 0 ? d->max_symbols_per_step
                                            : (W.type == PK_MODEL_TDT ? 10 : 5);
    if (W.type == PK_MODEL_EOU) {
        W.eou = d->eou_id >= 0 ? d->eou_id : d->vocab_size - 2;  // parakeet_eou.cpp:182
        W.eob = d->eob_id >= 0 ? d->eob_id : d->vocab_size - 1;  // parakeet_eou.cpp:183
        if (d->special_piece && d->n_vocab_pieces > 0)
            W.special.assign(d->special_piece, d->special_piece + d->n_vocab_pieces);
    } else {
        if (d->durations && d->num_durations > 0)
            W.durations.assign(d->durations, d->durations + d->num_durations);
    }
    bool ok = check(W.type == PK_MODEL_TDT || W.type == PK_MODEL_EOU, "bad model_type", err, errlen)
           && check(W.H > 0 && W.J > 0 && W.De > 0 && W.L > 0 && W.V1 > 1, "bad dims", err, errlen)
           && check(d->lstm != nullptr, "missing lstm layers", err, errlen)
           && check(W.blank >= 0 && W.blank < W.V1, "blank out of range", err, errlen)
           && check(W.type != PK_MODEL_TDT || W.Nd > 0, "TDT needs durations", err, errlen);
    if (ok) {
        ok = check(d->embed.ne0 == W.H && d->embed.ne1 >= W.V1, "embed shape", err, errlen)
          && check(shape_ok(d->joint_enc_w, W.De, W.J) && shape_ok(d->joint_enc_b, W.J, 1), "joint.enc shape", err, errlen)
          && check(shape_ok(d->joint_pred_w, W.H, W.J) && shape_ok(d->joint_pred_b, W.J, 1), "joint.pred shape", err, errlen)
          && check(d->joint_out_w.ne0 == W.J && d->joint_out_w.ne1 >= W.Vo && d->joint_out_b.ne0 >= W.Vo,
                   "joint.out shape", err, errlen);
        for (int l = 0; ok && l < W.L; ++l) {
            const pk_lstm_layer & ly = d->lstm[l];
            ok = check(shape_ok(ly.w_ih, W.H, 4 * W.H) && shape_ok(ly.w_hh, W.H, 4 * W.H)
                       && shape_ok(ly.b_ih, 4 * W.H, 1) && shape_ok(ly.b_hh, 4 * W.H, 1),
                       "lstm layer shape", err, errlen);
        }
    }
    std::string e;
    auto deq = [&](const pk_tensor & t, std::vector<float> & out, int64_t keep) {
        if (!ok) return;
        if (!dequantize(t, out, e)) { ok = false; check(false, e.c_str(), err, errlen); return; }
        if (keep >= 0 && (int64_t) out.size() > keep) out.resize((size_t) keep);
    };
    // tdt_prepare_runtime CPU branch, src/parakeet_tdt.cpp:620-639
    deq(d->embed, W.embed, (int64_t) W.V1 * W.H);
    W.lstm.resize((size_t) std::max(W.L, 0));
    for (int l = 0; ok && l < W.L; ++l) {
        deq(d->lstm[l].w_ih, W.lstm[(size_t) l].w_ih, -1);
        deq(d->lstm[l].w_hh, W.lstm[(size_t) l].w_hh, -1);
        deq(d->lstm[l].b_ih, W.lstm[(size_t) l].b_ih, -1);
        deq(d->lstm[l].b_hh, W.lstm[(size_t) l].b_hh, -1);
    }
    deq(d->joint_enc_w, W.enc_w, -1);
    deq(d->joint_enc_b, W.enc_b, -1);
    deq(d->joint_pred_w, W.pred_w, -1);
    deq(d->joint_pred_b, W.pred_b, -1);
    deq(d->joint_out_w, W.out_w, (int64_t) W.Vo * W.J);
    deq(d->joint_out_b, W.out_b, W.Vo);
    if (!ok) { delete m; return nullptr; }
    return m;
}

void orc_destroy(orc_model * m) { delete m; }

void orc_dims(const orc_model * m, int32_t * d) {
    d[0] = m->H; d[1] = m->J; d[2] = m->De; d[3] = m->L;
    d[4] = m->V1; d[5] = m->Vo; d[6] = m->Nd; d[7] = m->blank;
}

void orc_init_state(const orc_model * m, orc_state * st) {
    const orc_model & W = *m;
    const size_t n = (size_t) W.L * W.H;
    std::fill(st->h, st->h + n, 0.0f);
    std::fill(st->c, st->c + n, 0.0f);
    std::fill(st->pred, st->pred + W.H, 0.0f);
    st->symbols_this_step = 0;
    st->carry_frames = 0;                 // tdt_init_state :819
    st->last_token = -1;                  // eou_init_state :213
    st->segment_start_token = 0;          // eou_init_state :215
    Scratch s;
    const float * embed_row = W.embed.data() + (size_t) W.blank * W.H;   // :855 / eou :221
    lstm_step(W, embed_row, st->h, st->c, s);
    copy_pred(W, st);
    st->initialized = 1;
}

int32_t orc_tdt_decode_window(const orc_model * m, const float * enc, int32_t n_frames,
                              int32_t d_enc, int32_t max_symbols, orc_state * st,
                              int32_t * tokens, int32_t cap, int32_t * n_tokens,
                              int32_t * out_steps, orc_trace * tr) {
    const orc_model & W = *m;
    *out_steps = 0;                                             // :873
    if (d_enc != W.De) return 1;                                // :874-878
    if (n_frames <= 0) return 0;                                // :879
    if (!st->initialized) orc_init_state(m, st);                // :881-883
    const int V_p1 = W.V1, D_n = W.Nd, H = W.H;
    const int blank = W.blank;
    Scratch s;
    int t = 0;
    if (st->carry_frames > 0) {                                 // :907-910
        t = std::min(st->carry_frames, n_frames);
        st->carry_frames -= t;
    }
    int nt = *n_tokens;
    while (t < n_frames) {                                      // :919
        const float * enc_frame = enc + (size_t) t * d_enc;
        joint_step(W, enc_frame, st->pred, W.Vo, s);            // :931-932
        const int best_token = argmax_f32(s.logits.data(), V_p1);          // :933
        const int best_dur_idx = argmax_f32(s.logits.data() + V_p1, D_n);  // :934
        const int step = (*out_steps)++;                        // :936
        if (tr && step < tr->max_steps) {
            if (tr->logits) std::memcpy(tr->logits + (size_t) step * W.Vo, s.logits.data(), (size_t) W.Vo * 4);
            if (tr->token) tr->token[step] = best_token;
            if (tr->dur_idx) tr->dur_idx[step] = best_dur_idx;
            if (tr->margin_tok) tr->margin_tok[step] = top2_margin(s.logits.data(), V_p1);
            if (tr->margin_dur) tr->margin_dur[step] = top2_margin(s.logits.data() + V_p1, D_n);
            if (tr->frame) tr->frame[step] = t;
        }
        const int best_dur = W.durations.empty() ? best_dur_idx : W.durations[(size_t) best_dur_idx];  // :938-940
        if (best_token == blank) {                              // :942-946
            t += std::max(1, best_dur);
            st->symbols_this_step = 0;
            trace_state(W, st, tr, step);
            continue;
        }
        if (nt >= cap) return -1;
        tokens[nt++] = best_token;                              // :948
        const float * embed_row = W.embed.data() + (size_t) best_token * H;   // :955-960
        lstm_step(W, embed_row, st->h, st->c, s);
        copy_pred(W, st);
        trace_state(W, st, tr, step);
        ++st->symbols_this_step;                                // :963-967
        if (best_dur > 0 || st->symbols_this_step >= max_symbols) {
            t += std::max(1, best_dur);
            st->symbols_this_step = 0;
        }
    }
    st->carry_frames = std::max(0, t - n_frames);               // :979
    *n_tokens = nt;
    return 0;
}

int32_t orc_eou_decode_window(const orc_model * m, const float * enc, int32_t n_frames,
                              int32_t d_enc, int32_t max_symbols, orc_state * st,
                              int32_t * tokens, int32_t cap, int32_t * n_tokens,
                              int32_t * bounds, int32_t bounds_cap, int32_t * n_bounds,
                              int32_t * out_steps, orc_trace * tr) {
    const orc_model & W = *m;
    if (d_enc != W.De) return 1;                                // parakeet_eou.cpp:241-245
    if (!st->initialized) orc_init_state(m, st);                // :246-248
    const int H = W.H, L = W.L, V_p1 = W.V1;
    const int blank = W.blank, eou = W.eou, eob = W.eob;
    const int max_syms = std::max(1, max_symbols);              // :256
    Scratch s;
    *out_steps = 0;                                             // :264
    int nt = *n_tokens;
    int nb = n_bounds ? *n_bounds : 0;
    const int n_vocab = (int) W.special.size();
    for (int t = 0; t < n_frames; ++t) {                        // :267
        const float * enc_frame = enc + (size_t) t * d_enc;
        st->symbols_this_step = 0;
        while (st->symbols_this_step < max_syms) {              // :271
            joint_step(W, enc_frame, st->pred, V_p1, s);
            const int step = (*out_steps)++;
            const int best = argmax_f32(s.logits.data(), V_p1); // :277
            if (tr && step < tr->max_steps) {
                if (tr->logits) std::memcpy(tr->logits + (size_t) step * V_p1, s.logits.data(), (size_t) V_p1 * 4);
                if (tr->token) tr->token[step] = best;
                if (tr->dur_idx) tr->dur_idx[step] = 0;
                if (tr->margin_tok) tr->margin_tok[step] = top2_margin(s.logits.data(), V_p1);
                if (tr->margin_dur) tr->margin_dur[step] = INFINITY;
                if (tr->frame) tr->frame[step] = t;
            }
            if (best == blank) { trace_state(W, st, tr, step); break; }     // :278
            if (best == eob) { trace_state(W, st, tr, step); break; }       // :283
            if (best == eou) {                                              // :292-311
                if (nt > st->segment_start_token) {
                    if (bounds) {
                        if (nb >= bounds_cap) return -1;
                        bounds[nb] = nt;
                    }
                    ++nb;
                    st->segment_start_token = nt;
                }
                std::fill(st->h, st->h + (size_t) L * H, 0.0f);
                std::fill(st->c, st->c + (size_t) L * H, 0.0f);
                st->last_token = blank;
                const float * embed_row = W.embed.data() + (size_t) blank * H;
                lstm_step(W, embed_row, st->h, st->c, s);
                copy_pred(W, st);
                trace_state(W, st, tr, step);
                break;
            }
            if (best >= 0 && best < n_vocab && W.special[(size_t) best]) {  // :315-319
                trace_state(W, st, tr, step);
                break;
            }
            if (nt >= cap) return -1;
            tokens[nt++] = best;                                            // :322
            const float * embed_row = W.embed.data() + (size_t) best * H;
            lstm_step(W, embed_row, st->h, st->c, s);
            copy_pred(W, st);
            trace_state(W, st, tr, step);
            st->last_token = best;
            ++st->symbols_this_step;
        }
    }
    *n_tokens = nt;
    if (n_bounds) *n_bounds = nb;
    return 0;
}

double orc_decode_batch(const orc_model * m, const float * enc, const int64_t * frame_off,
                        const int32_t * n_frames, int32_t B, int32_t max_symbols,
                        int32_t n_threads, int32_t * tokens, const int64_t * tok_region,
                        int32_t * n_tok, int32_t * steps,
                        int32_t * bounds, const int64_t * bound_region, int32_t * n_bounds,
                        double * ms) {
    const orc_model & W = *m;
    if (B <= 0) return 0.0;
    if (n_threads <= 0) n_threads = (int32_t) std::max(1u, std::thread::hardware_concurrency());
    n_threads = std::min(n_threads, B);
    const int msym = max_symbols > 0 ? max_symbols : W.max_sym;
    std::atomic<int> next{0};
    std::atomic<int> failed{0};
    auto worker = [&]() {
        std::vector<float> h((size_t) W.L * W.H), c((size_t) W.L * W.H), p((size_t) W.H);
        for (;;) {
            const int b = next.fetch_add(1);
            if (b >= B) break;
            const auto t0 = std::chrono::steady_clock::now();
            orc_state st{h.data(), c.data(), p.data(), 0, 0, 0, -1, 0};
            const int T = n_frames[b];
            const float * e = enc + (size_t) frame_off[b] * W.De;
            int32_t nt = 0, ns = 0, nb = 0;
            const int32_t cap = (int32_t) ((int64_t) T * std::max(1, msym));
            int32_t rc;
            if (W.type == PK_MODEL_TDT) {
                // tdt_greedy_decode, src/parakeet_tdt.cpp:983-1005 (fresh state)
                rc = orc_tdt_decode_window(m, e, T, W.De, msym, &st, tokens + tok_region[b], cap,
                                           &nt, &ns, nullptr);
            } else {
                // eou_greedy_decode, src/parakeet_eou.cpp:338-387
                int32_t bcap = bounds ? std::max(T, 0) : 0;
                rc = orc_eou_decode_window(m, e, T, W.De, msym, &st, tokens + tok_region[b], cap, &nt,
                                           bounds ? bounds + bound_region[b] : nullptr, bcap, &nb,
                                           &ns, nullptr);
            }
            if (rc != 0) failed.store(1);
            n_tok[b] = nt;
            if (steps) steps[b] = ns;
            if (n_bounds) n_bounds[b] = nb;
            if (ms) ms[b] = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        }
    };
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<std::thread> pool;
    for (int i = 1; i < n_threads; ++i) pool.emplace_back(worker);
    worker();
    for (auto & th : pool) th.join();
    const double wall = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return failed.load() ? -1.0 : wall;
}

// ctc_greedy_decode_window (src/parakeet_ctc.cpp:1831-1865): per frame the
// first index of the maximum (`>` scan from index 0), emitted when it is not
// blank and differs from the previous frame's; prev carries across windows.
int32_t orc_ctc_greedy_window(const float * logits, int32_t n_frames, int32_t vocab_size, int32_t blank_id,
                              int32_t * prev, int32_t * tokens, int32_t cap, int32_t * n_tokens,
                              int32_t * first_frame) {
    int32_t p = *prev;
    for (int32_t t = 0; t < n_frames; ++t) {
        const float * row = logits + (size_t) t * vocab_size;
        int32_t best = 0;
        float best_score = row[0];
        for (int32_t i = 1; i < vocab_size; ++i) {
            if (row[i] > best_score) { best_score = row[i]; best = i; }
        }
        if (best != blank_id && best != p) {
            if (*n_tokens >= cap) return -1;
            if (first_frame) first_frame[*n_tokens] = t;
            tokens[(*n_tokens)++] = best;
        }
        p = best;
    }
    *prev = p;
    return 0;
}

// detokenize (src/sentencepiece_bpe.cpp:9-37): skip ids outside the vocabulary
// and the blank / bos / eos / pad ids; copy each piece with every E2 96 81
// (U+2581) replaced by one space; drop the text's leading spaces.
int64_t orc_detokenize(const uint8_t * bytes, const int64_t * offsets, int32_t n_pieces, int32_t blank_id,
                       int32_t bos_id, int32_t eos_id, int32_t pad_id, const int32_t * tokens, int64_t n_tokens,
                       char * text, int64_t cap) {
    std::string out;
    for (int64_t k = 0; k < n_tokens; ++k) {
        const int32_t id = tokens[k];
        if (id < 0 || id >= n_pieces) continue;
        if (id == blank_id || id == bos_id || id == eos_id || id == pad_id) continue;
        const int64_t a = offsets[id], e = offsets[id + 1];
        for (int64_t i = a; i < e;) {
            if (bytes[i] == 0xE2 && i + 2 < e && bytes[i + 1] == 0x96 && bytes[i + 2] == 0x81) {
                out.push_back(' ');
                i += 3;
            } else {
                out.push_back((char) bytes[i]);
                ++i;
            }
        }
    }
    size_t start = 0;
    while (start < out.size() && out[start] == ' ') ++start;
    const int64_t n = (int64_t) (out.size() - start);
    if (text) std::memcpy(text, out.data() + start, (size_t) std::min<int64_t>(n, cap));
    return n;
}

}  // extern "C"
