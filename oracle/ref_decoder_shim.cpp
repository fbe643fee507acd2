// ref_decoder_shim.cpp -- TEST INFRASTRUCTURE ONLY: C entry points around the
// reference's OWN decoder, src/parakeet_tdt.cpp and src/parakeet_eou.cpp
// compiled unchanged where they lie (Makefile target `ref`) against the
// host-only ggml stand-in in ggml_host/. The result, oracle/_ref/libref_decoder.so,
// is the pin for the CPU restatement in oracle.cpp and the "reference" CPU
// baseline; the product library never links or calls it.
//
// It builds a parakeet::ParakeetCtcModel from a pk_model_desc (the same raw
// GGUF blocks the product takes), with tensors in host memory and a backend that
// reports a CPU device, so tdt_prepare_runtime takes its CPU branch
// (src/parakeet_tdt.cpp:620) and eou_prepare_runtime dequantizes as it always
// does (src/parakeet_eou.cpp:172-204). Decoding then calls the reference's own
// tdt_decode_window / eou_decode_window / tdt_greedy_decode / eou_greedy_decode.

#include "parakeet_eou.h"
#include "parakeet_log.h"
#include "parakeet_tdt.h"

#include "ggml.h"
#include "ggml-backend.h"

#include "parakeet_cuda.h"
#include "ref_model.hpp"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

ggml_backend_t ggml_host_cpu_backend();

// ParakeetCtcModel's accessors live in the reference's parakeet_ctc.cpp (the
// GGUF loader and encoder, not built here); the decoder needs only the backend.
namespace parakeet {
ggml_backend_t ParakeetCtcModel::backend_active() const { return ggml_host_cpu_backend(); }
ggml_context * ParakeetCtcModel::weights_ctx() const { return nullptr; }

// parakeet_log.cpp's log_impl forwards to a ggml log hook; stderr is enough here.
void log_impl(enum ggml_log_level, const char * fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    std::vfprintf(stderr, fmt, ap);
    va_end(ap);
}
}  // namespace parakeet

struct ref_model : refmodel::Model {
    parakeet::TdtRuntimeWeights tdt;
    parakeet::EouRuntimeWeights eou;
};

struct ref_state {
    parakeet::TdtDecodeState tdt;
    parakeet::EouDecodeState eou;
};

extern "C" {

ref_model * ref_create(const pk_model_desc * d, char * err, int32_t errlen) {
    auto fail = [&](const char * msg) -> ref_model * {
        if (err && errlen > 0) std::snprintf(err, (size_t) errlen, "%s", msg);
        return nullptr;
    };
    if (!d) return fail("null descriptor");
    auto m = std::make_unique<ref_model>();
    m->fill(*d);
    parakeet::ParakeetCtcModel & M = m->model;
    try {
        if (m->is_tdt) {
            if (parakeet::tdt_prepare_runtime(M, m->tdt) != 0) return fail("tdt_prepare_runtime failed");
            if (m->tdt.use_graphs) return fail("tdt_prepare_runtime chose the graph branch");
        } else {
            if (parakeet::eou_prepare_runtime(M, m->eou) != 0) return fail("eou_prepare_runtime failed");
        }
    } catch (const std::exception & e) {
        return fail(e.what());
    }
    return m.release();
}

void ref_destroy(ref_model * m) { delete m; }

ref_state * ref_state_new(void) { return new ref_state(); }
void ref_state_free(ref_state * s) { delete s; }

// State after the last window: h, c ([L][H]) and pred ([H]) when the state is
// initialised; ints = {symbols_this_step, initialized, carry_frames (TDT),
// last_token (EOU), segment_start_token (EOU)}.
void ref_state_get(const ref_model * m, const ref_state * s, float * h, float * c, float * pred, int32_t * ints) {
    if (m->is_tdt) {
        const auto & st = s->tdt;
        if (h) std::copy(st.h_state.begin(), st.h_state.end(), h);
        if (c) std::copy(st.c_state.begin(), st.c_state.end(), c);
        if (pred) std::copy(st.pred_out.begin(), st.pred_out.end(), pred);
        ints[0] = st.symbols_this_step; ints[1] = st.initialized; ints[2] = st.carry_frames;
        ints[3] = -1; ints[4] = 0;
    } else {
        const auto & st = s->eou;
        if (h) std::copy(st.h_state.begin(), st.h_state.end(), h);
        if (c) std::copy(st.c_state.begin(), st.c_state.end(), c);
        if (pred) std::copy(st.pred_out.begin(), st.pred_out.end(), pred);
        ints[0] = st.symbols_this_step; ints[1] = st.initialized; ints[2] = 0;
        ints[3] = st.last_token; ints[4] = st.segment_start_token;
    }
}

// One tdt_decode_window / eou_decode_window call. tokens[0 .. *n_tokens) on
// entry is the caller's running token list (the reference's out_tokens); the
// window's tokens are appended and *n_tokens updated. EOU boundaries of this
// window go to bounds (count in *n_bounds). Returns the reference's rc, or -1
// when `cap` / `bounds_cap` is too small.
int32_t ref_decode_window(ref_model * m, ref_state * s, const float * enc, int32_t n_frames, int32_t d_enc,
                          int32_t max_symbols, int32_t * tokens, int32_t cap, int32_t * n_tokens, int32_t * steps,
                          int32_t * bounds, int32_t bounds_cap, int32_t * n_bounds) {
    std::vector<int32_t> out(tokens, tokens + *n_tokens);
    int out_steps = 0;
    int rc;
    try {
        if (m->is_tdt) {
            parakeet::TdtDecodeOptions o;
            o.max_symbols_per_step = max_symbols > 0 ? max_symbols : m->max_symbols;
            rc = parakeet::tdt_decode_window(m->model, m->tdt, enc, n_frames, d_enc, o, s->tdt, out, out_steps);
            if (n_bounds) *n_bounds = 0;
        } else {
            parakeet::EouDecodeOptions o;
            o.max_symbols_per_step = max_symbols > 0 ? max_symbols : m->max_symbols;
            std::vector<parakeet::EouSegmentBoundary> seg;
            rc = parakeet::eou_decode_window(m->model, m->eou, enc, n_frames, d_enc, o, s->eou, out, seg, out_steps);
            if ((int32_t) seg.size() > bounds_cap) return -1;
            for (size_t i = 0; i < seg.size(); ++i) bounds[i] = seg[i].token_index;
            if (n_bounds) *n_bounds = (int32_t) seg.size();
        }
    } catch (const std::exception & e) {
        std::fprintf(stderr, "ref_decode_window: %s\n", e.what());
        return -2;
    }
    if ((int64_t) out.size() > cap) return -1;
    std::copy(out.begin() + *n_tokens, out.end(), tokens + *n_tokens);
    *n_tokens = (int32_t) out.size();
    if (steps) *steps = out_steps;
    return rc;
}

// B fresh utterances through the reference's own tdt_greedy_decode /
// eou_greedy_decode, one utterance per host thread at a time (weights shared
// read-only: the CPU branch never writes them). Same layout as
// orc_decode_batch; ms[b] = the reference's decode_ms. Returns the batch's
// wall time in ms, negative on error.
double ref_decode_batch(ref_model * m, const float * enc, const int64_t * frame_off, const int32_t * n_frames,
                        int32_t B, int32_t max_symbols, int32_t n_threads, int32_t * tokens,
                        const int64_t * tok_region, int32_t * n_tok, int32_t * steps, int32_t * bounds,
                        const int64_t * bound_region, int32_t * n_bounds, double * ms) {
    if (B <= 0) return 0.0;
    if (n_threads <= 0) n_threads = (int32_t) std::max(1u, std::thread::hardware_concurrency());
    n_threads = std::min(n_threads, B);
    const int msym = max_symbols > 0 ? max_symbols : m->max_symbols;
    const int De = m->is_tdt ? m->tdt.D_enc : m->eou.D_enc;
    std::atomic<int> next{0};
    std::atomic<int> failed{0};
    auto worker = [&]() {
        for (;;) {
            const int b = next.fetch_add(1);
            if (b >= B) break;
            const float * e = enc + (size_t) frame_off[b] * De;
            const int T = n_frames[b];
            try {
                if (m->is_tdt) {
                    parakeet::TdtDecodeOptions o;
                    o.max_symbols_per_step = msym;
                    parakeet::TdtDecodeResult r;
                    if (parakeet::tdt_greedy_decode(m->model, m->tdt, e, T, De, o, r) != 0) failed.store(1);
                    std::copy(r.token_ids.begin(), r.token_ids.end(), tokens + tok_region[b]);
                    n_tok[b] = (int32_t) r.token_ids.size();
                    if (steps) steps[b] = r.steps;
                    if (n_bounds) n_bounds[b] = 0;
                    if (ms) ms[b] = r.decode_ms;
                } else {
                    parakeet::EouDecodeOptions o;
                    o.max_symbols_per_step = msym;
                    parakeet::EouDecodeResult r;
                    if (parakeet::eou_greedy_decode(m->model, m->eou, e, T, De, o, r) != 0) failed.store(1);
                    std::copy(r.token_ids.begin(), r.token_ids.end(), tokens + tok_region[b]);
                    n_tok[b] = (int32_t) r.token_ids.size();
                    if (steps) steps[b] = r.steps;
                    if (bounds && n_bounds) {
                        for (size_t i = 0; i < r.segments.size(); ++i)
                            bounds[bound_region[b] + (int64_t) i] = r.segments[i].token_index;
                        n_bounds[b] = (int32_t) r.segments.size();
                    }
                    if (ms) ms[b] = r.decode_ms;
                }
            } catch (const std::exception &) {
                failed.store(1);
            }
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

}  // extern "C"
