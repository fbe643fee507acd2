// parakeet_decoder_cuda.cpp -- C++17 drop-in for parakeet.cpp's decoder dispatch.
//
// Implements, with the reference's exact declarations and return codes, the
// functions of src/parakeet_tdt.h:185-205 and src/parakeet_eou.h:82-107 on top of
// libparakeet_cuda's C ABI (include/parakeet_cuda.h), so that the Engine's call
// sites (src/parakeet_engine.cpp:155-166, 273-297, 403-457, 809-838) compile and
// behave unchanged:
//
//   tdt_prepare_runtime / tdt_init_state / tdt_decode_window / tdt_greedy_decode
//   eou_prepare_runtime / eou_init_state / eou_decode_window / eou_greedy_decode
//   TdtRuntimeWeights' move constructor, move assignment and destructor
//
// Build it in place of src/parakeet_tdt.cpp and src/parakeet_eou.cpp, against the
// reference's headers (and ggml's), and link libparakeet_cuda.so. The device is
// CUDA device 0 unless PARAKEET_CUDA_DEVICE names another.
//
// State handling mirrors the reference's CPU branch: TdtDecodeState /
// EouDecodeState keep h, c and pred_out on the host between windows (the caller
// owns them, as in the reference), so each window uploads the state, runs the
// device step loop for the window and downloads the new state. Weights are read
// once at prepare time through ggml_backend_tensor_get (so they may live on any
// ggml backend) and repacked onto the GPU by pk_create.
//
// A runtime's device context is found by the runtime's address: a
// TdtRuntimeWeights carries it across moves (its special members are defined
// here); an EouRuntimeWeights (a plain aggregate in the reference) must stay at
// the address eou_prepare_runtime saw, as the Engine's does.

#include "parakeet_eou.h"
#include "parakeet_tdt.h"
#include "sentencepiece_bpe.h"

#include "ggml.h"
#include "ggml-backend.h"

#include "parakeet_cuda.h"

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

namespace parakeet {
namespace {

// ---- device contexts by runtime address ---------------------------------------

struct Device {
    pk_ctx * ctx = nullptr;
    pk_stream * stream = nullptr;   // the one window-decoding stream of this runtime
};

std::mutex g_mu;
std::map<const void *, Device> g_dev;

Device * find_device(const void * rt) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_dev.find(rt);
    return it == g_dev.end() ? nullptr : &it->second;
}

void drop_device(const void * rt) {
    Device d;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_dev.find(rt);
        if (it == g_dev.end()) return;
        d = it->second;
        g_dev.erase(it);
    }
    if (d.stream) pk_stream_destroy(d.stream);
    if (d.ctx) pk_destroy(d.ctx);
}

void move_device(const void * from, const void * to) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_dev.find(from);
    if (it == g_dev.end()) return;
    g_dev[to] = it->second;
    g_dev.erase(it);
}

int device_index() {
    const char * s = std::getenv("PARAKEET_CUDA_DEVICE");
    return s ? std::atoi(s) : 0;
}

// ---- GGUF tensors -> the C descriptor -------------------------------------------

// Raw blocks of one ggml tensor, fetched from its backend.
struct Raw {
    std::vector<uint8_t> bytes;
    pk_tensor t{};
};

bool fetch(const ggml_tensor * g, Raw & r) {
    if (!g) return false;
    const size_t n = ggml_nbytes(g);
    r.bytes.resize(n);
    ggml_backend_tensor_get(g, r.bytes.data(), 0, n);
    r.t.data = r.bytes.data();
    r.t.type = (int32_t) g->type;
    r.t.ne0 = g->ne[0];
    r.t.ne1 = g->ne[1];
    r.t.nbytes = n;
    return true;
}

template <class Weights>
struct DescBuilder {
    std::vector<Raw> raws;
    std::vector<pk_lstm_layer> lstm;
    std::vector<int32_t> durations;
    std::vector<uint8_t> special;
    pk_model_desc d{};

    bool build(const ParakeetCtcModel & model, const Weights & w, bool tdt) {
        const int L = (int) w.lstm.size();
        raws.resize(7 + 4 * (size_t) L);
        size_t k = 0;
        auto take = [&](const ggml_tensor * g, pk_tensor & dst) {
            Raw & r = raws[k++];
            if (!fetch(g, r)) return false;
            dst = r.t;
            return true;
        };
        if (!take(w.predict_embed, d.embed) || !take(w.joint_enc_w, d.joint_enc_w) ||
            !take(w.joint_enc_b, d.joint_enc_b) || !take(w.joint_pred_w, d.joint_pred_w) ||
            !take(w.joint_pred_b, d.joint_pred_b) || !take(w.joint_out_w, d.joint_out_w) ||
            !take(w.joint_out_b, d.joint_out_b))
            return false;
        lstm.resize((size_t) L);
        for (int l = 0; l < L; ++l) {
            if (!take(w.lstm[l].w_ih, lstm[l].w_ih) || !take(w.lstm[l].w_hh, lstm[l].w_hh) ||
                !take(w.lstm[l].b_ih, lstm[l].b_ih) || !take(w.lstm[l].b_hh, lstm[l].b_hh))
                return false;
        }
        const EncoderConfig & cfg = model.encoder_cfg;
        d.model_type = tdt ? PK_MODEL_TDT : PK_MODEL_EOU;
        d.d_enc = cfg.d_model;
        d.pred_hidden = tdt ? cfg.tdt_pred_hidden : cfg.eou_pred_hidden;
        d.joint_hidden = tdt ? cfg.tdt_joint_hidden : cfg.eou_joint_hidden;
        d.n_layers = L;
        d.vocab_size = model.vocab_size;
        d.blank_id = model.blank_id;
        if (tdt) {
            // the reference indexes model.tdt_durations when present, else uses the index itself
            durations = model.tdt_durations;
            if (durations.empty())
                for (int i = 0; i < cfg.tdt_num_durations; ++i) durations.push_back(i);
            d.num_durations = (int32_t) durations.size();
            d.durations = durations.data();
            d.max_symbols_per_step = 10;   // TdtDecodeOptions default; each call passes its own
        } else {
            d.eou_id = model.eou_id;
            d.eob_id = model.eob_id;
            d.max_symbols_per_step = cfg.eou_max_symbols_per_step;
            // pieces shaped "<...>" are skipped without emission (parakeet_eou.cpp:315-319)
            special.resize(model.vocab.pieces.size());
            for (size_t i = 0; i < special.size(); ++i) {
                const std::string & p = model.vocab.pieces[i];
                special[i] = (!p.empty() && p.front() == '<' && p.back() == '>') ? 1 : 0;
            }
            d.n_vocab_pieces = (int32_t) special.size();
            d.special_piece = special.empty() ? nullptr : special.data();
        }
        d.lstm = lstm.data();
        return true;
    }
};

template <class Weights>
int prepare(const ParakeetCtcModel & model, const Weights & w, bool tdt, const void * key) {
    DescBuilder<Weights> b;
    if (!w.predict_embed || w.lstm.empty() || !w.joint_out_w || !b.build(model, w, tdt)) {
        std::fprintf(stderr, "%s_prepare_runtime: GGUF is missing decoder tensors\n", tdt ? "tdt" : "eou");
        return 2;
    }
    Device dev;
    if (pk_create(&b.d, device_index(), &dev.ctx) != PK_OK) {
        std::fprintf(stderr, "%s_prepare_runtime: %s\n", tdt ? "tdt" : "eou", pk_last_error());
        return 3;
    }
    if (pk_stream_create(dev.ctx, &dev.stream) != PK_OK) {
        std::fprintf(stderr, "%s_prepare_runtime: %s\n", tdt ? "tdt" : "eou", pk_last_error());
        pk_destroy(dev.ctx);
        return 3;
    }
    drop_device(key);
    std::lock_guard<std::mutex> lk(g_mu);
    g_dev[key] = dev;
    return 0;
}

// Host state <-> the device stream.
template <class State>
pk_stream_state view(State & st, int32_t carry, int32_t last, int32_t segstart) {
    pk_stream_state v{};
    v.h = st.h_state.data();
    v.c = st.c_state.data();
    v.pred_out = st.pred_out.data();
    v.symbols_this_step = st.symbols_this_step;
    v.carry_frames = carry;
    v.initialized = st.initialized ? 1 : 0;
    v.last_token = last;
    v.segment_start_token = segstart;
    return v;
}

template <class State>
bool fresh_state(pk_stream * s, int L, int H, State & st) {
    st.h_state.assign((size_t) L * H, 0.0f);
    st.c_state.assign((size_t) L * H, 0.0f);
    st.pred_out.assign((size_t) H, 0.0f);
    pk_stream_state v = view(st, 0, -1, 0);
    return pk_stream_reset(s) == PK_OK && pk_stream_get_state(s, &v) == PK_OK;
}

std::string trim_spaces(const std::string & s) {
    const size_t a = s.find_first_not_of(" \t\r\n");
    if (a == std::string::npos) return std::string();
    const size_t b = s.find_last_not_of(" \t\r\n");
    return s.substr(a, b - a + 1);
}

}  // namespace

// ---- TDT (src/parakeet_tdt.h:185-205) -----------------------------------------------

TdtRuntimeWeights::TdtRuntimeWeights(TdtRuntimeWeights && o) noexcept { *this = std::move(o); }

TdtRuntimeWeights & TdtRuntimeWeights::operator=(TdtRuntimeWeights && o) noexcept {
    if (this == &o) return *this;
    drop_device(this);
    H_pred = o.H_pred; H_joint = o.H_joint; D_enc = o.D_enc; V_plus_1 = o.V_plus_1; V_out = o.V_out;
    L = o.L; num_durations = o.num_durations;
    weights = o.weights; o.weights = nullptr;
    backend = o.backend; o.backend = nullptr;
    n_threads = o.n_threads;
    use_graphs = o.use_graphs;
    move_device(&o, this);
    return *this;
}

TdtRuntimeWeights::~TdtRuntimeWeights() { drop_device(this); }

int tdt_prepare_runtime(const ParakeetCtcModel & model, TdtRuntimeWeights & W) {
    W = TdtRuntimeWeights{};
    const EncoderConfig & cfg = model.encoder_cfg;
    W.H_pred = cfg.tdt_pred_hidden;
    W.H_joint = cfg.tdt_joint_hidden;
    W.D_enc = cfg.d_model;
    W.L = cfg.tdt_pred_rnn_layers;
    W.num_durations = cfg.tdt_num_durations;
    W.V_plus_1 = (int) model.vocab_size + 1;
    W.V_out = W.V_plus_1 + W.num_durations;
    const int rc = prepare(model, model.tdt, true, &W);
    if (rc != 0) return rc;
    W.weights = &model.tdt;
    W.use_graphs = true;   // decoding runs on the device
    return 0;
}

void tdt_init_state(TdtRuntimeWeights & W, int /*blank_id: the model's, set at prepare*/, TdtDecodeState & state) {
    Device * d = find_device(&W);
    state.symbols_this_step = 0;
    state.carry_frames = 0;
    if (!d || !fresh_state(d->stream, W.L, W.H_pred, state))
        throw std::runtime_error(std::string("tdt_init_state: ") + (d ? pk_last_error() : "runtime not prepared"));
    state.initialized = true;
}

int tdt_decode_window(const ParakeetCtcModel & model, TdtRuntimeWeights & W, const float * encoder_out_window,
                      int n_frames, int D_enc, const TdtDecodeOptions & opts, TdtDecodeState & state,
                      std::vector<int32_t> & out_tokens, int & out_steps) {
    out_steps = 0;
    if (D_enc != W.D_enc) {
        std::fprintf(stderr, "tdt_decode_window: encoder d_model mismatch (%d vs %d)\n", D_enc, W.D_enc);
        return 1;
    }
    if (n_frames <= 0) return 0;
    if (!state.initialized) tdt_init_state(W, (int) model.blank_id, state);
    Device * d = find_device(&W);
    if (!d) return 6;
    pk_stream_state v = view(state, state.carry_frames, -1, 0);
    if (pk_stream_set_state(d->stream, &v) != PK_OK) return 7;
    const int msym = std::max(1, opts.max_symbols_per_step);
    std::vector<int32_t> toks((size_t) n_frames * msym);
    int32_t nt = 0, steps = 0;
    if (pk_stream_window(d->stream, encoder_out_window, 0, n_frames, D_enc, msym, (int32_t) out_tokens.size(),
                         toks.data(), (int32_t) toks.size(), &nt, &steps, nullptr, 0, nullptr) != PK_OK) {
        std::fprintf(stderr, "tdt_decode_window: %s\n", pk_last_error());
        return 7;
    }
    if (pk_stream_get_state(d->stream, &v) != PK_OK) return 9;
    out_tokens.insert(out_tokens.end(), toks.begin(), toks.begin() + nt);
    out_steps = steps;
    state.symbols_this_step = v.symbols_this_step;
    state.carry_frames = v.carry_frames;
    return 0;
}

int tdt_greedy_decode(const ParakeetCtcModel & model, TdtRuntimeWeights & W, const float * encoder_out, int T_enc,
                      int D_enc, const TdtDecodeOptions & opts, TdtDecodeResult & result) {
    const auto t0 = std::chrono::steady_clock::now();
    TdtDecodeState state;
    result.token_ids.clear();
    result.token_ids.reserve(T_enc);
    if (int rc = tdt_decode_window(model, W, encoder_out, T_enc, D_enc, opts, state, result.token_ids, result.steps);
        rc != 0)
        return rc;
    result.text = detokenize(model.vocab, result.token_ids);
    const auto t1 = std::chrono::steady_clock::now();
    result.decode_ms = std::chrono::duration_cast<std::chrono::microseconds>(t1 - t0).count() / 1000.0;
    return 0;
}

// ---- EOU (src/parakeet_eou.h:82-107) ------------------------------------------------

int eou_prepare_runtime(const ParakeetCtcModel & model, EouRuntimeWeights & W) {
    if (model.model_type != ParakeetModelType::EOU) return 1;
    const EncoderConfig & cfg = model.encoder_cfg;
    W.H_pred = cfg.eou_pred_hidden;
    W.H_joint = cfg.eou_joint_hidden;
    W.D_enc = cfg.d_model;
    W.L = cfg.eou_pred_rnn_layers;
    W.V_plus_1 = (int) model.vocab_size + 1;
    W.blank_id = (int) model.blank_id;
    W.eou_id = model.eou_id >= 0 ? model.eou_id : (int) model.vocab_size - 2;
    W.eob_id = model.eob_id >= 0 ? model.eob_id : (int) model.vocab_size - 1;
    return prepare(model, model.eou, false, &W);
}

void eou_init_state(const EouRuntimeWeights & W, EouDecodeState & state) {
    Device * d = find_device(&W);
    state.last_token = -1;
    state.symbols_this_step = 0;
    state.segment_start_token = 0;
    if (!d || !fresh_state(d->stream, W.L, W.H_pred, state))
        throw std::runtime_error(std::string("eou_init_state: ") + (d ? pk_last_error() : "runtime not prepared"));
    state.last_token = -1;   // the reference primes on blank without recording it
    state.initialized = true;
}

int eou_decode_window(const ParakeetCtcModel & /*model*/, const EouRuntimeWeights & W,
                      const float * encoder_out_window, int n_frames, int D_enc, const EouDecodeOptions & opts,
                      EouDecodeState & state, std::vector<int32_t> & out_tokens,
                      std::vector<EouSegmentBoundary> & out_segments, int & out_steps) {
    if (D_enc != W.D_enc) {
        std::fprintf(stderr, "eou_decode_window: encoder d_model mismatch (%d vs %d)\n", D_enc, W.D_enc);
        return 1;
    }
    if (!state.initialized) eou_init_state(W, state);
    out_steps = 0;
    Device * d = find_device(&W);
    if (!d) return 6;
    pk_stream_state v = view(state, 0, state.last_token, state.segment_start_token);
    if (pk_stream_set_state(d->stream, &v) != PK_OK) return 7;
    const int msym = std::max(1, opts.max_symbols_per_step);
    const int nf = std::max(0, n_frames);
    std::vector<int32_t> toks((size_t) std::max(1, nf * msym)), bnd((size_t) std::max(1, nf));
    int32_t nt = 0, steps = 0, nb = 0;
    if (pk_stream_window(d->stream, encoder_out_window, 0, nf, D_enc, msym, (int32_t) out_tokens.size(),
                         toks.data(), (int32_t) toks.size(), &nt, &steps, bnd.data(), (int32_t) bnd.size(),
                         &nb) != PK_OK) {
        std::fprintf(stderr, "eou_decode_window: %s\n", pk_last_error());
        return 7;
    }
    if (pk_stream_get_state(d->stream, &v) != PK_OK) return 9;
    out_tokens.insert(out_tokens.end(), toks.begin(), toks.begin() + nt);
    for (int32_t i = 0; i < nb; ++i) {
        EouSegmentBoundary s;
        s.token_index = bnd[(size_t) i];
        s.is_eou_flush = true;
        out_segments.push_back(s);
    }
    out_steps = steps;
    state.symbols_this_step = v.symbols_this_step;
    state.last_token = v.last_token;
    state.segment_start_token = v.segment_start_token;
    return 0;
}

int eou_greedy_decode(const ParakeetCtcModel & model, const EouRuntimeWeights & W, const float * encoder_out,
                      int T_enc, int D_enc, const EouDecodeOptions & opts, EouDecodeResult & result) {
    const auto t0 = std::chrono::steady_clock::now();
    EouDecodeState state;
    result.token_ids.clear();
    result.segments.clear();
    result.token_ids.reserve(T_enc);
    if (int rc = eou_decode_window(model, W, encoder_out, T_enc, D_enc, opts, state, result.token_ids,
                                   result.segments, result.steps);
        rc != 0)
        return rc;
    result.eou_count = (int) result.segments.size();
    // segments joined with '\n', each detokenized and trimmed (parakeet_eou.cpp:338-387)
    int seg_start = 0;
    std::string out_text;
    for (size_t i = 0; i <= result.segments.size(); ++i) {
        const int seg_end = i < result.segments.size() ? result.segments[i].token_index : (int) result.token_ids.size();
        if (seg_end <= seg_start) {
            seg_start = seg_end;
            continue;
        }
        const std::vector<int32_t> seg(result.token_ids.begin() + seg_start, result.token_ids.begin() + seg_end);
        const std::string t = trim_spaces(detokenize(model.vocab, seg));
        if (!t.empty()) {
            if (!out_text.empty()) out_text += "\n";
            out_text += t;
        }
        seg_start = seg_end;
    }
    result.text = std::move(out_text);
    const auto t1 = std::chrono::steady_clock::now();
    result.decode_ms = std::chrono::duration_cast<std::chrono::microseconds>(t1 - t0).count() / 1000.0;
    return 0;
}

}  // namespace parakeet
