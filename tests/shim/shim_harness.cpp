// shim_harness.cpp -- TEST HARNESS: drives the C++17 drop-in decoder
// (parakeet.cpp_b200/shim/parakeet_decoder_cuda.cpp) exactly as the reference's
// Engine does -- parakeet::tdt_prepare_runtime / eou_prepare_runtime on a
// ParakeetCtcModel, then tdt_decode_window / eou_decode_window window by window
// with the state carried in TdtDecodeState / EouDecodeState, or the
// *_greedy_decode calls -- and exposes that through a few C functions for pytest
// (tests/test_shim.py), which compares the results with the CPU oracle.
//
// The model's tensors are host-memory ggml tensors of the host-only ggml
// stand-in (oracle/ggml_host/), so the shim reads them through the same
// ggml_nbytes / ggml_backend_tensor_get calls it makes against real ggml.

#include "parakeet_eou.h"
#include "parakeet_tdt.h"

#include "ref_model.hpp"

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace {

struct Harness : refmodel::Model {
    parakeet::TdtRuntimeWeights tdt;
    parakeet::EouRuntimeWeights eou;
    parakeet::TdtDecodeState tdt_state;
    parakeet::EouDecodeState eou_state;
    std::vector<int32_t> tokens;      // the running out_tokens of the stream
};

}  // namespace

extern "C" {

// rc of tdt_prepare_runtime / eou_prepare_runtime in *rc; NULL on failure.
void * shim_open(const pk_model_desc * d, int32_t * rc) {
    auto * h = new Harness();
    h->fill(*d);
    *rc = h->is_tdt ? parakeet::tdt_prepare_runtime(h->model, h->tdt) : parakeet::eou_prepare_runtime(h->model, h->eou);
    if (*rc != 0) {
        delete h;
        return nullptr;
    }
    return h;
}

void shim_close(void * p) { delete static_cast<Harness *>(p); }

// tdt_init_state / eou_init_state on the harness's stream state (also clears its token list).
int32_t shim_init_state(void * p) {
    auto * h = static_cast<Harness *>(p);
    h->tokens.clear();
    try {
        if (h->is_tdt) parakeet::tdt_init_state(h->tdt, (int) h->model.blank_id, h->tdt_state);
        else parakeet::eou_init_state(h->eou, h->eou_state);
    } catch (const std::exception & e) {
        std::fprintf(stderr, "shim_init_state: %s\n", e.what());
        return -1;
    }
    return 0;
}

// One decode_window call on the harness's stream. New tokens are appended to the
// harness's running list; tokens (cap entries) receives the whole list, *n_tokens its
// length; bounds receives this window's EOU boundaries. Returns the call's rc.
int32_t shim_window(void * p, const float * enc, int32_t n_frames, int32_t d_enc, int32_t max_symbols,
                    int32_t * tokens, int32_t cap, int32_t * n_tokens, int32_t * steps,
                    int32_t * bounds, int32_t bounds_cap, int32_t * n_bounds) {
    auto * h = static_cast<Harness *>(p);
    int rc, st = 0;
    if (n_bounds) *n_bounds = 0;
    if (h->is_tdt) {
        parakeet::TdtDecodeOptions o;
        o.max_symbols_per_step = max_symbols;
        rc = parakeet::tdt_decode_window(h->model, h->tdt, enc, n_frames, d_enc, o, h->tdt_state, h->tokens, st);
    } else {
        parakeet::EouDecodeOptions o;
        o.max_symbols_per_step = max_symbols;
        std::vector<parakeet::EouSegmentBoundary> seg;
        rc = parakeet::eou_decode_window(h->model, h->eou, enc, n_frames, d_enc, o, h->eou_state, h->tokens, seg, st);
        if ((int32_t) seg.size() > bounds_cap) return -1;
        for (size_t i = 0; i < seg.size(); ++i) bounds[i] = seg[i].token_index;
        if (n_bounds) *n_bounds = (int32_t) seg.size();
    }
    if ((int32_t) h->tokens.size() > cap) return -1;
    std::memcpy(tokens, h->tokens.data(), h->tokens.size() * 4);
    *n_tokens = (int32_t) h->tokens.size();
    if (steps) *steps = st;
    return rc;
}

// State after the last window: h, c [L][H], pred [H]; ints = {symbols_this_step,
// initialized, carry_frames, last_token, segment_start_token}.
void shim_state(void * p, float * hs, float * cs, float * ps, int32_t * ints) {
    auto * h = static_cast<Harness *>(p);
    auto put = [&](const auto & st) {
        std::memcpy(hs, st.h_state.data(), st.h_state.size() * 4);
        std::memcpy(cs, st.c_state.data(), st.c_state.size() * 4);
        std::memcpy(ps, st.pred_out.data(), st.pred_out.size() * 4);
        ints[0] = st.symbols_this_step;
        ints[1] = st.initialized;
    };
    if (h->is_tdt) {
        put(h->tdt_state);
        ints[2] = h->tdt_state.carry_frames; ints[3] = -1; ints[4] = 0;
    } else {
        put(h->eou_state);
        ints[2] = 0; ints[3] = h->eou_state.last_token; ints[4] = h->eou_state.segment_start_token;
    }
}

// tdt_greedy_decode / eou_greedy_decode of one utterance; text is the result's text.
int32_t shim_greedy(void * p, const float * enc, int32_t T, int32_t d_enc, int32_t max_symbols, int32_t * tokens,
                    int32_t cap, int32_t * n_tokens, int32_t * steps, int32_t * bounds, int32_t bounds_cap,
                    int32_t * n_bounds, char * text, int32_t text_cap, int32_t * text_len) {
    auto * h = static_cast<Harness *>(p);
    std::vector<int32_t> ids;
    std::string txt;
    int rc, st = 0;
    if (n_bounds) *n_bounds = 0;
    if (h->is_tdt) {
        parakeet::TdtDecodeOptions o;
        o.max_symbols_per_step = max_symbols;
        parakeet::TdtDecodeResult r;
        rc = parakeet::tdt_greedy_decode(h->model, h->tdt, enc, T, d_enc, o, r);
        ids = r.token_ids; st = r.steps; txt = r.text;
    } else {
        parakeet::EouDecodeOptions o;
        o.max_symbols_per_step = max_symbols;
        parakeet::EouDecodeResult r;
        rc = parakeet::eou_greedy_decode(h->model, h->eou, enc, T, d_enc, o, r);
        ids = r.token_ids; st = r.steps; txt = r.text;
        if ((int32_t) r.segments.size() > bounds_cap) return -1;
        for (size_t i = 0; i < r.segments.size(); ++i) bounds[i] = r.segments[i].token_index;
        if (n_bounds) *n_bounds = (int32_t) r.segments.size();
    }
    if ((int32_t) ids.size() > cap) return -1;
    std::memcpy(tokens, ids.data(), ids.size() * 4);
    *n_tokens = (int32_t) ids.size();
    if (steps) *steps = st;
    *text_len = (int32_t) txt.size();
    std::memcpy(text, txt.data(), std::min<size_t>(txt.size(), (size_t) std::max(0, text_cap)));
    return rc;
}

}  // extern "C"
