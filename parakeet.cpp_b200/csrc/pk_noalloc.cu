// pk_noalloc.cu -- pk_decode_noalloc: greedy decode of one utterance without any
// device allocation during the call.
//
// Some callers cannot call cudaMalloc while they decode: a process that runs
// under a fixed device-memory budget (its allocator refuses new device memory
// after start-up), or a latency-critical audio thread for which cudaMalloc's
// implicit device synchronisation and possible failure are unacceptable. This
// entry point serves them: every buffer the enc-proj GEMM and the persistent
// step loop need beyond the caller's inputs and outputs lives in one
// file-scope device array of fixed size (PK_NOALLOC_SCRATCH_BYTES), which every
// GPU that loads the library holds until the process exits.
//
// In host code `g_scratch` is only a host-side stand-in for the array: giving
// it to a kernel would fault (or, where the GPU can reach host memory, use the
// wrong memory). Host code therefore passes the array's device address, looked
// up once per device with cudaGetSymbolAddress while that device is current.
// pk_create does that look-up (noalloc_prepare below), so this file's module --
// and with it the array -- is loaded when the context is made, not lazily at the
// first call, and it runs one 1-frame decode on the CUDA-core loop this entry
// point uses, so that kernel's local memory is sized then too. The call itself
// runs the f32 CUDA-core enc-proj and step loop whatever the context's math
// mode. All calls share the array and it keeps the last call's contents: the
// init kernel below clears everything that must start at zero, and calls that
// overlap on the GPU race with each other.

#include "pk_internal.h"

#include <mutex>

namespace pk {
namespace {

constexpr int kNaMaxDevices = 64;
constexpr int kNaMaxDim = 1024;   // joint_hidden and pred_hidden limit

static __device__ __align__(256) unsigned char g_scratch[PK_NOALLOC_SCRATCH_BYTES];

std::mutex g_mu;
unsigned char * g_addr[kNaMaxDevices] = {};

struct Layout {
    size_t encp, h, c, predp, hid, ust, keys, live, livef, emit, ctl, bar, tstart, finish, tokregion,
        bndregion, frameoff, bnd, total;
};

size_t up256(size_t x) { return (x + 255) & ~(size_t) 255; }

Layout layout(int J, int H, int L) {
    Layout o{};
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t at = off; off = up256(off + bytes); return at; };
    o.encp = take((size_t) PK_NOALLOC_MAX_FRAMES * J * 4);
    o.h = take((size_t) 2 * L * H * 4);
    o.c = take((size_t) L * H * 4);
    o.predp = take((size_t) J * 4);
    o.hid = take((size_t) J * 4);
    o.ust = take(kUst * 4);
    o.keys = take(4 * 8);   // two alternating argmax key buffers
    o.live = take(2 * 4);
    o.livef = take(2 * 8);
    o.emit = take(2 * 4);
    o.ctl = take(kCtl * 4);
    o.bar = take(8 * 4);
    o.tstart = take(8);
    o.finish = take(8);
    o.tokregion = take(8);
    o.bndregion = take(8);
    o.frameoff = take(8);
    o.bnd = take((size_t) PK_NOALLOC_MAX_FRAMES * 4);
    o.total = off;
    return o;
}

// Sets up the one-utterance loop state: clears what must start at zero and
// writes the initial lists (fresh utterance: init LSTM step on the blank token).
__global__ void noalloc_init_kernel(unsigned char * base, Layout o, int T, int blank, int fresh) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int32_t * ust = reinterpret_cast<int32_t *>(base + o.ust);
    for (int i = 0; i < kUst; ++i) ust[i] = 0;
    ust[U_LAST] = -1;
    ust[U_NFRAMES] = T;
    int32_t * ctl = reinterpret_cast<int32_t *>(base + o.ctl);
    for (int i = 0; i < kCtl; ++i) ctl[i] = 0;
    int32_t * live = reinterpret_cast<int32_t *>(base + o.live);
    live[0] = 0;
    live[1] = 0;
    int64_t * livef = reinterpret_cast<int64_t *>(base + o.livef);
    livef[0] = 0;   // frame row of the live utterance: frame_offset 0 + t 0
    livef[1] = 0;
    ctl[C_NLIVE0] = T > 0 ? 1 : 0;
    int32_t * emit = reinterpret_cast<int32_t *>(base + o.emit);
    emit[0] = 0;
    emit[1] = blank | (1 << 31);
    ctl[C_NEMIT] = fresh ? 1 : 0;
    unsigned long long * keys = reinterpret_cast<unsigned long long *>(base + o.keys);
    for (int i = 0; i < 4; ++i) keys[i] = 0ull;
    unsigned * bar = reinterpret_cast<unsigned *>(base + o.bar);
    for (int i = 0; i < 8; ++i) bar[i] = 0u;
    *reinterpret_cast<unsigned long long *>(base + o.finish) = 0ull;
    *reinterpret_cast<int64_t *>(base + o.tokregion) = 0;
    *reinterpret_cast<int64_t *>(base + o.bndregion) = 0;
    *reinterpret_cast<int64_t *>(base + o.frameoff) = 0;
}

__global__ void noalloc_finish_kernel(const unsigned char * base, Layout o, int32_t * n_tokens,
                                      int32_t * steps) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const int32_t * ust = reinterpret_cast<const int32_t *>(base + o.ust);
    *n_tokens = ust[U_NTOK];
    *steps = ust[U_STEPS];
}

pk_status na_fail(pk_status s, const char * msg) { return set_error(s, msg); }

// Device address of g_scratch on `device` (which must be current).
pk_status scratch_address(int device, unsigned char ** out) {
    if (device < 0 || device >= kNaMaxDevices) return PK_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_addr[device] == nullptr) {
        void * p = nullptr;
        if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || p == nullptr) return PK_ERR_CUDA;
        g_addr[device] = static_cast<unsigned char *>(p);
    }
    *out = g_addr[device];
    return PK_OK;
}

}  // namespace

// Called by pk_create with the context's device current: looks up the scratch
// array's device address, which loads this file's module (and with it the
// array's device memory) now instead of at the first pk_decode_noalloc call, when
// CUDA loads modules lazily (its default since 12.2).
pk_status noalloc_prepare(int device) {
    unsigned char * base = nullptr;
    if (scratch_address(device, &base) != PK_OK) return PK_ERR_CUDA;
    cudaFuncAttributes a{};
    if (cudaFuncGetAttributes(&a, noalloc_init_kernel) != cudaSuccess ||
        cudaFuncGetAttributes(&a, noalloc_finish_kernel) != cudaSuccess)
        return PK_ERR_CUDA;
    return PK_OK;
}

}  // namespace pk

extern "C" PK_API pk_status pk_decode_noalloc(pk_ctx * ctx, const float * enc, int32_t n_frames,
                                              int32_t d_enc, int32_t max_symbols, int32_t * tokens,
                                              int32_t tokens_cap, int32_t * n_tokens, int32_t * steps) {
    using namespace pk;
    if (!ctx || !tokens || !n_tokens || !steps || (n_frames > 0 && !enc))
        return na_fail(PK_ERR_INVALID, "pk_decode_noalloc: null argument");
    CtxView v;
    ctx_view(ctx, &v);
    if (d_enc != v.De) return na_fail(PK_ERR_DMODEL, "pk_decode_noalloc: encoder d_model mismatch");
    if ((reinterpret_cast<uintptr_t>(enc) | reinterpret_cast<uintptr_t>(tokens) | reinterpret_cast<uintptr_t>(n_tokens) |
         reinterpret_cast<uintptr_t>(steps)) & 3u)
        return na_fail(PK_ERR_INVALID, "pk_decode_noalloc: device pointers must be 4-byte aligned");
    if (n_frames < 0 || n_frames > PK_NOALLOC_MAX_FRAMES)
        return na_fail(PK_ERR_INVALID, "pk_decode_noalloc: n_frames outside [0, PK_NOALLOC_MAX_FRAMES = 4096]");
    if (v.J > kNaMaxDim || v.H > kNaMaxDim)
        return na_fail(PK_ERR_INVALID, "pk_decode_noalloc: joint_hidden / pred_hidden above 1024");
    const int msym = max_symbols > 0 ? max_symbols : v.max_sym;
    if ((int64_t) tokens_cap < (int64_t) n_frames * (msym > 0 ? msym : 1))
        return na_fail(PK_ERR_CAPACITY, "pk_decode_noalloc: tokens_cap < n_frames * max_symbols_per_step");
    const Layout o = layout(v.J, v.H, v.L);
    if (o.total > PK_NOALLOC_SCRATCH_BYTES)
        return na_fail(PK_ERR_INVALID, "pk_decode_noalloc: model too large for the static scratch array");
    int prev_device = -1;
    if (cudaGetDevice(&prev_device) != cudaSuccess) prev_device = -1;
    if (cudaSetDevice(v.device) != cudaSuccess) return na_fail(PK_ERR_CUDA, "pk_decode_noalloc: cudaSetDevice failed");
    // the caller's current device comes back on every return from here on
    struct Restore {
        int d;
        ~Restore() { if (d >= 0) cudaSetDevice(d); }
    } restore{prev_device};
    unsigned char * base = nullptr;
    if (scratch_address(v.device, &base) != PK_OK)
        return na_fail(PK_ERR_CUDA, "pk_decode_noalloc: cudaGetSymbolAddress of the scratch array failed");
    cudaStream_t s = v.stream;
    // tdt_decode_window initialises only when n_frames > 0 (parakeet_tdt.cpp:879-883);
    // eou_decode_window always does (parakeet_eou.cpp:246-248).
    const int fresh = (!v.is_tdt || n_frames > 0) ? 1 : 0;
    noalloc_init_kernel<<<1, 32, 0, s>>>(base, o, n_frames, v.blank, fresh);
    if (cudaGetLastError() != cudaSuccess) return na_fail(PK_ERR_CUDA, "pk_decode_noalloc: init launch failed");
    float * encp = reinterpret_cast<float *>(base + o.encp);
    if (n_frames > 0 && launch_encproj_f32(enc, n_frames, v.De, v.enc_w, v.enc_b, v.J, encp, s) != cudaSuccess)
        return na_fail(PK_ERR_CUDA, "pk_decode_noalloc: enc-proj launch failed");
    LoopParams P{};
    P.H = v.H; P.J = v.J; P.L = v.L; P.V1 = v.V1; P.Vo = v.Vo; P.Nd = v.Nd; P.blank = v.blank;
    P.eou = v.eou; P.eob = v.eob; P.is_tdt = v.is_tdt; P.max_sym = msym; P.B = 1;
    P.n_special = v.n_special; P.chunk = v.chunk; P.ldx = v.ldx; P.timeout_ns = v.timeout_ns;
    P.max_iters = n_frames * ((msym > 0 ? msym : 1) + 1) + 2;
    P.embed = v.embed;
    for (int l = 0; l < kMaxLayers; ++l) {
        P.w_ih[l] = v.w_ih[l]; P.w_hh[l] = v.w_hh[l]; P.b_ih[l] = v.b_ih[l]; P.b_hh[l] = v.b_hh[l];
    }
    P.pred_w = v.pred_w; P.pred_b = v.pred_b; P.out_w = v.out_w; P.out_b = v.out_b;
    P.durations = v.durations; P.special = v.special;
    P.encp = encp;
    P.frame_off = reinterpret_cast<const int64_t *>(base + o.frameoff);
    P.h = reinterpret_cast<float *>(base + o.h);
    P.c = reinterpret_cast<float *>(base + o.c);
    P.predp = reinterpret_cast<float *>(base + o.predp);
    P.hid = reinterpret_cast<float *>(base + o.hid);
    P.ust = reinterpret_cast<int32_t *>(base + o.ust);
    P.keys = reinterpret_cast<unsigned long long *>(base + o.keys);
    P.live = reinterpret_cast<int32_t *>(base + o.live);
    P.live_frame = reinterpret_cast<int64_t *>(base + o.livef);
    P.emit = reinterpret_cast<int32_t *>(base + o.emit);
    P.ctl = reinterpret_cast<int32_t *>(base + o.ctl);
    P.bar = reinterpret_cast<unsigned *>(base + o.bar);
    P.t_start = reinterpret_cast<unsigned long long *>(base + o.tstart);
    P.finish_ns = reinterpret_cast<unsigned long long *>(base + o.finish);
    P.tok_out = tokens;
    P.tok_region = reinterpret_cast<const int64_t *>(base + o.tokregion);
    P.bnd_out = reinterpret_cast<int32_t *>(base + o.bnd);
    P.bnd_region = reinterpret_cast<const int64_t *>(base + o.bndregion);
    if (launch_step_loop(P, v.grid, v.smem, s) != cudaSuccess)
        return na_fail(PK_ERR_CUDA, "pk_decode_noalloc: step-loop launch failed");
    noalloc_finish_kernel<<<1, 32, 0, s>>>(base, o, n_tokens, steps);
    if (cudaGetLastError() != cudaSuccess) return na_fail(PK_ERR_CUDA, "pk_decode_noalloc: finish launch failed");
    int32_t err = 0;
    if (cudaMemcpyAsync(&err, base + o.ctl + C_ERR * 4, sizeof(err), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return na_fail(PK_ERR_CUDA, "pk_decode_noalloc: device error during the decode");
    if (err != 0) return na_fail((pk_status) err, "pk_decode_noalloc: step loop reported a device error");
    return PK_OK;
}
