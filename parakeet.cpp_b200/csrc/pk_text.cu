// pk_text.cu -- the two steps beside the token loop: CTC greedy decode
// (src/parakeet_ctc.cpp:1820-1865) and SentencePiece detokenize
// (src/sentencepiece_bpe.cpp:9-37), batched over utterances on the GPU.
//
// Both are byte / integer work bound by HBM (the logits) or by latency (the
// texts): plain coalesced loads, block scans for the compactions, one CTA per
// utterance where an utterance's output order matters.

#include "pk_internal.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

namespace pk {
namespace {

constexpr int kTxtThreads = 256;

struct Buf {
    void * p = nullptr;
    size_t cap = 0;
    cudaError_t ensure(size_t bytes) {
        if (bytes <= cap && (p != nullptr || bytes == 0)) return cudaSuccess;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        const size_t want = bytes + bytes / 8 + 256;
        const cudaError_t e = cudaMalloc(&p, want);
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

pk_status cuda_fail(cudaError_t e, const char * where) {
    char msg[256];
    std::snprintf(msg, sizeof(msg), "%s: %s", where, cudaGetErrorString(e));
    return set_error(e == cudaErrorMemoryAllocation ? PK_ERR_OOM : PK_ERR_CUDA, msg);
}

#define TX_CK(call, where)                              \
    do {                                                \
        const cudaError_t e_ = (call);                  \
        if (e_ != cudaSuccess) return cuda_fail(e_, where); \
    } while (0)

// Block-wide exclusive scan of one int per thread (kTxtThreads threads).
__device__ __forceinline__ int block_scan(int v, int * s_warp, int & total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const int w = lane < kTxtThreads / 32 ? s_warp[lane] : 0;
        int y = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int z = __shfl_up_sync(0xFFFFFFFFu, y, o);
            if (lane >= o) y += z;
        }
        if (lane < kTxtThreads / 32) s_warp[lane] = y - w;
        if (lane == kTxtThreads / 32 - 1) s_warp[kTxtThreads / 32] = y;
    }
    __syncthreads();
    total = s_warp[kTxtThreads / 32];
    const int r = x - v + s_warp[warp];
    __syncthreads();
    return r;
}

// Exclusive scan of counts[0..n) into offs[0..n] (offs[n] = total), one block.
__global__ void __launch_bounds__(kTxtThreads) scan_offsets_kernel(const int * counts, int n, int64_t * offs) {
    __shared__ int s_warp[kTxtThreads / 32 + 1];
    int64_t base = 0;
    for (int c0 = 0; c0 < n; c0 += kTxtThreads) {
        const int i = c0 + (int) threadIdx.x;
        const int v = i < n ? counts[i] : 0;
        int tot = 0;
        const int ex = block_scan(v, s_warp, tot);
        if (i < n) offs[i] = base + ex;
        base += tot;
    }
    if (threadIdx.x == 0) offs[n] = base;
}

// ---- CTC greedy ----------------------------------------------------------------

// One warp per frame: the argmax of ctc_greedy_decode_window's `>` scan from
// index 0 (parakeet_ctc.cpp:1843-1853). Lanes scan strided indices in increasing
// order, skipping NaNs (a NaN never compares greater); lanes merge by value, then
// lower index. If row[0] is NaN the scan's running best stays NaN and index 0 wins.
__global__ void __launch_bounds__(kTxtThreads) ctc_argmax_kernel(const float * __restrict__ logits,
                                                                 long long frames, int V,
                                                                 int * __restrict__ best) {
    const int lane = threadIdx.x & 31;
    const long long wid = ((long long) blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long) gridDim.x * blockDim.x) >> 5;
    for (long long f = wid; f < frames; f += nw) {
        const float * row = logits + f * (long long) V;
        bool has = false;
        float bv = 0.0f;
        int bi = 0;
        int i = lane;
        // eight independent loads in flight per lane
        for (; i + 7 * 32 < V; i += 8 * 32) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = __ldcs(row + i + u * 32);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (v[u] == v[u] && (!has || v[u] > bv)) { has = true; bv = v[u]; bi = i + u * 32; }
            }
        }
        for (; i < V; i += 32) {
            const float v = __ldcs(row + i);
            if (v == v && (!has || v > bv)) { has = true; bv = v; bi = i; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const int oh = __shfl_xor_sync(0xFFFFFFFFu, has ? 1 : 0, o);
            const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
            const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
            if (oh && (!has || ov > bv || (ov == bv && oi < bi))) { has = true; bv = ov; bi = oi; }
        }
        if (lane == 0) {
            const float r0 = row[0];
            best[f] = (r0 != r0 || !has) ? 0 : bi;
        }
    }
}

// One CTA per utterance: a frame emits its argmax when it is not blank and
// differs from the previous frame's (the window's first frame compares with
// prev_in); emitted tokens and their frames go compacted to the utterance's
// region (n_frames entries at region_off: at most one token per frame).
__global__ void __launch_bounds__(kTxtThreads) ctc_collapse_kernel(const int * __restrict__ best,
                                                                   const int64_t * __restrict__ frame_off,
                                                                   const int * __restrict__ n_frames,
                                                                   const int64_t * __restrict__ region_off,
                                                                   const int * __restrict__ prev_in, int blank,
                                                                   int * __restrict__ rtok, int * __restrict__ rframe,
                                                                   int * __restrict__ counts, int * __restrict__ prev_out) {
    __shared__ int s_warp[kTxtThreads / 32 + 1];
    const int b = blockIdx.x;
    const int64_t f0 = frame_off[b], r0 = region_off[b];
    const int n = n_frames[b];
    const int p0 = prev_in[b];
    int count = 0;
    for (int t0 = 0; t0 < n; t0 += kTxtThreads) {
        const int t = t0 + (int) threadIdx.x;
        int tok = 0, e = 0;
        if (t < n) {
            tok = best[f0 + t];
            const int prev = t == 0 ? p0 : best[f0 + t - 1];
            e = (tok != blank && tok != prev) ? 1 : 0;
        }
        int tot = 0;
        const int pos = block_scan(e, s_warp, tot);
        if (e) {
            rtok[r0 + count + pos] = tok;
            rframe[r0 + count + pos] = t;
        }
        count += tot;
    }
    if (threadIdx.x == 0) {
        counts[b] = count;
        prev_out[b] = n > 0 ? best[f0 + n - 1] : p0;
    }
}

// Compaction of the per-utterance regions into one array (offsets from the scan).
__global__ void __launch_bounds__(kTxtThreads) gather_regions_kernel(const int * __restrict__ src,
                                                                     const int64_t * __restrict__ src_off,
                                                                     const int64_t * __restrict__ dst_off,
                                                                     int * __restrict__ dst) {
    const int b = blockIdx.x;
    const int64_t s = src_off[b], d = dst_off[b], n = dst_off[b + 1] - dst_off[b];
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) dst[d + i] = src[s + i];
}

// ---- detokenize --------------------------------------------------------------

// Decoded vocabulary on the device: piece v's bytes (U+2581 already turned into
// a space, specials and nothing else emptied) at bytes[off[v] .. off[v] + len[v]),
// lead[v] = its leading spaces (len[v] when all of it is spaces).
struct VocabDev {
    const unsigned char * bytes;
    const int64_t * off;
    const int * len;
    const int * lead;
    int n;
};

__device__ __forceinline__ int piece_of(const VocabDev & v, int tok) { return (tok >= 0 && tok < v.n) ? tok : -1; }

// One CTA per utterance: the text length after dropping its leading spaces, and
// how many leading bytes to drop (the first non-space byte of the joined pieces).
__global__ void __launch_bounds__(kTxtThreads) detok_measure_kernel(VocabDev v, const int * __restrict__ tokens,
                                                                    const int64_t * __restrict__ tok_off,
                                                                    int * __restrict__ text_len,
                                                                    int * __restrict__ lead_out) {
    __shared__ int s_warp[kTxtThreads / 32 + 1];
    __shared__ int s_first;
    const int b = blockIdx.x;
    const int64_t t0 = tok_off[b], nt = tok_off[b + 1] - t0;
    if (threadIdx.x == 0) s_first = 0x7FFFFFFF;
    int base = 0;
    for (int64_t c0 = 0; c0 < nt; c0 += kTxtThreads) {
        const int64_t i = c0 + threadIdx.x;
        int len = 0, ld = 0;
        if (i < nt) {
            const int pc = piece_of(v, tokens[t0 + i]);
            if (pc >= 0) { len = v.len[pc]; ld = v.lead[pc]; }
        }
        int tot = 0;
        const int pos = block_scan(len, s_warp, tot);
        if (ld < len) atomicMin(&s_first, base + pos + ld);
        base += tot;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const int first = min(s_first, base);
        lead_out[b] = first;
        text_len[b] = base - first;
    }
}

// One CTA per utterance: each thread copies its tokens' decoded bytes to their
// place in the joined text, minus the dropped leading spaces.
__global__ void __launch_bounds__(kTxtThreads) detok_write_kernel(VocabDev v, const int * __restrict__ tokens,
                                                                  const int64_t * __restrict__ tok_off,
                                                                  const int * __restrict__ lead,
                                                                  const int64_t * __restrict__ text_off,
                                                                  unsigned char * __restrict__ text) {
    __shared__ int s_warp[kTxtThreads / 32 + 1];
    const int b = blockIdx.x;
    const int64_t t0 = tok_off[b], nt = tok_off[b + 1] - t0;
    const int drop = lead[b];
    unsigned char * out = text + text_off[b];
    int base = 0;
    for (int64_t c0 = 0; c0 < nt; c0 += kTxtThreads) {
        const int64_t i = c0 + threadIdx.x;
        int len = 0, pc = -1;
        if (i < nt) {
            pc = piece_of(v, tokens[t0 + i]);
            if (pc >= 0) len = v.len[pc];
        }
        int tot = 0;
        const int pos = base + block_scan(len, s_warp, tot);
        for (int j = 0; j < len; ++j) {
            const int g = pos + j;
            if (g >= drop) out[g - drop] = v.bytes[v.off[pc] + j];
        }
        base += tot;
    }
}

}  // namespace
}  // namespace pk

// ---- C ABI ---------------------------------------------------------------------

struct pk_ctc {
    int device = 0;
    cudaStream_t stream = nullptr;
    int V = 0, blank = 0;
    pk::Buf logits, best, foff, roff, nfr, prev_in, prev_out, rtok, rframe, counts, offs, otok, oframe;
};

struct pk_vocab {
    int device = 0;
    cudaStream_t stream = nullptr;
    int n = 0;
    pk::Buf bytes, off, len, lead, tokens, tokoff, textlen, textlead, textoff, text;
};

namespace {

bool on_sm100(int device) {
    cudaDeviceProp p{};
    return cudaGetDeviceProperties(&p, device) == cudaSuccess && p.major == 10;
}

}  // namespace

extern "C" PK_API pk_status pk_ctc_create(int device, int32_t vocab_size, int32_t blank_id, pk_ctc ** out) {
    using namespace pk;
    if (!out) return set_error(PK_ERR_INVALID, "pk_ctc_create: null output");
    *out = nullptr;
    if (vocab_size <= 0 || blank_id < 0 || blank_id >= vocab_size)
        return set_error(PK_ERR_INVALID, "pk_ctc_create: vocab_size must be > 0 and blank_id in [0, vocab_size)");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n || !on_sm100(device))
        return set_error(PK_ERR_NO_DEVICE, "pk_ctc_create: no sm_100 device with that index");
    TX_CK(cudaSetDevice(device), "pk_ctc_create: cudaSetDevice");
    pk_ctc * c = new pk_ctc();
    c->device = device;
    c->V = vocab_size;
    c->blank = blank_id;
    const cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "pk_ctc_create: stream");
    }
    *out = c;
    return PK_OK;
}

extern "C" PK_API void pk_ctc_destroy(pk_ctc * c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (pk::Buf * b : {&c->logits, &c->best, &c->foff, &c->roff, &c->nfr, &c->prev_in, &c->prev_out, &c->rtok, &c->rframe,
                        &c->counts, &c->offs, &c->otok, &c->oframe})
        b->release();
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

extern "C" PK_API pk_status pk_ctc_greedy(pk_ctc * c, const float * logits, int32_t logits_on_device,
                                          const int64_t * frame_offsets, const int32_t * n_frames, int32_t B,
                                          int32_t * prev_inout, int32_t * tokens, int64_t tokens_cap,
                                          int64_t * token_offsets, int32_t * first_frame, int64_t * tokens_needed) {
    using namespace pk;
    if (!c || B < 0 || (B > 0 && (!frame_offsets || !n_frames || !prev_inout || !token_offsets)) ||
        (tokens_cap > 0 && !tokens) || tokens_cap < 0)
        return set_error(PK_ERR_INVALID, "pk_ctc_greedy: null argument or negative size");
    if (B == 0) {
        if (token_offsets) token_offsets[0] = 0;
        if (tokens_needed) *tokens_needed = 0;
        return PK_OK;
    }
    // utterance frame ranges: inside [0, frames) of the logits array, non-negative
    int64_t frames = 0;
    std::vector<int64_t> roff((size_t) B);   // each utterance's output region (its frame count)
    int64_t rtotal = 0;
    for (int b = 0; b < B; ++b) {
        if (n_frames[b] < 0 || frame_offsets[b] < 0)
            return set_error(PK_ERR_INVALID, "pk_ctc_greedy: negative frame offset or count");
        frames = std::max<int64_t>(frames, frame_offsets[b] + n_frames[b]);
        roff[b] = rtotal;
        rtotal += n_frames[b];
    }
    if (logits_on_device && (reinterpret_cast<uintptr_t>(logits) & 3u))
        return set_error(PK_ERR_INVALID, "pk_ctc_greedy: device logits must be 4-byte aligned");
    if (frames > 0 && !logits) return set_error(PK_ERR_INVALID, "pk_ctc_greedy: null logits");
    TX_CK(cudaSetDevice(c->device), "pk_ctc_greedy: cudaSetDevice");
    cudaStream_t s = c->stream;
    const size_t fb = (size_t) std::max<int64_t>(frames, 1);
    const float * dlog = logits;
    if (!logits_on_device && frames > 0) {
        TX_CK(c->logits.ensure(fb * c->V * 4), "pk_ctc_greedy: alloc");
        TX_CK(cudaMemcpyAsync(c->logits.p, logits, (size_t) frames * c->V * 4, cudaMemcpyHostToDevice, s),
              "pk_ctc_greedy: logits copy");
        dlog = c->logits.as<float>();
    }
    const size_t rb = (size_t) std::max<int64_t>(rtotal, 1);
    TX_CK(c->best.ensure(fb * 4), "pk_ctc_greedy: alloc");
    TX_CK(c->rtok.ensure(rb * 4), "pk_ctc_greedy: alloc");
    TX_CK(c->rframe.ensure(rb * 4), "pk_ctc_greedy: alloc");
    TX_CK(c->otok.ensure(rb * 4), "pk_ctc_greedy: alloc");
    TX_CK(c->oframe.ensure(rb * 4), "pk_ctc_greedy: alloc");
    TX_CK(c->roff.ensure((size_t) B * 8), "pk_ctc_greedy: alloc");
    TX_CK(c->foff.ensure((size_t) B * 8), "pk_ctc_greedy: alloc");
    TX_CK(c->nfr.ensure((size_t) B * 4), "pk_ctc_greedy: alloc");
    TX_CK(c->prev_in.ensure((size_t) B * 4), "pk_ctc_greedy: alloc");
    TX_CK(c->prev_out.ensure((size_t) B * 4), "pk_ctc_greedy: alloc");
    TX_CK(c->counts.ensure((size_t) B * 4), "pk_ctc_greedy: alloc");
    TX_CK(c->offs.ensure((size_t) (B + 1) * 8), "pk_ctc_greedy: alloc");
    TX_CK(cudaMemcpyAsync(c->foff.p, frame_offsets, (size_t) B * 8, cudaMemcpyHostToDevice, s), "pk_ctc_greedy: copy");
    TX_CK(cudaMemcpyAsync(c->roff.p, roff.data(), (size_t) B * 8, cudaMemcpyHostToDevice, s), "pk_ctc_greedy: copy");
    TX_CK(cudaMemcpyAsync(c->nfr.p, n_frames, (size_t) B * 4, cudaMemcpyHostToDevice, s), "pk_ctc_greedy: copy");
    TX_CK(cudaMemcpyAsync(c->prev_in.p, prev_inout, (size_t) B * 4, cudaMemcpyHostToDevice, s), "pk_ctc_greedy: copy");
    if (frames > 0) {
        const long long warps = frames;
        const int blocks = (int) std::min<long long>((warps + 7) / 8, 148LL * 8);
        ctc_argmax_kernel<<<blocks, kTxtThreads, 0, s>>>(dlog, frames, c->V, c->best.as<int>());
        TX_CK(cudaGetLastError(), "pk_ctc_greedy: argmax launch");
    }
    ctc_collapse_kernel<<<B, kTxtThreads, 0, s>>>(c->best.as<int>(), c->foff.as<int64_t>(), c->nfr.as<int>(),
                                                  c->roff.as<int64_t>(), c->prev_in.as<int>(), c->blank, c->rtok.as<int>(),
                                                  c->rframe.as<int>(), c->counts.as<int>(), c->prev_out.as<int>());
    TX_CK(cudaGetLastError(), "pk_ctc_greedy: collapse launch");
    scan_offsets_kernel<<<1, kTxtThreads, 0, s>>>(c->counts.as<int>(), B, c->offs.as<int64_t>());
    TX_CK(cudaGetLastError(), "pk_ctc_greedy: scan launch");
    TX_CK(cudaMemcpyAsync(token_offsets, c->offs.p, (size_t) (B + 1) * 8, cudaMemcpyDeviceToHost, s),
          "pk_ctc_greedy: offsets copy");
    TX_CK(cudaStreamSynchronize(s), "pk_ctc_greedy: sync");
    const int64_t total = token_offsets[B];
    if (tokens_needed) *tokens_needed = total;
    if (total > tokens_cap) {
        char msg[160];
        std::snprintf(msg, sizeof(msg), "pk_ctc_greedy: %lld tokens > tokens_cap %lld", (long long) total,
                      (long long) tokens_cap);
        return set_error(PK_ERR_CAPACITY, msg);
    }
    gather_regions_kernel<<<B, kTxtThreads, 0, s>>>(c->rtok.as<int>(), c->roff.as<int64_t>(), c->offs.as<int64_t>(),
                                                    c->otok.as<int>());
    if (first_frame)
        gather_regions_kernel<<<B, kTxtThreads, 0, s>>>(c->rframe.as<int>(), c->roff.as<int64_t>(),
                                                        c->offs.as<int64_t>(), c->oframe.as<int>());
    TX_CK(cudaGetLastError(), "pk_ctc_greedy: gather launch");
    if (total > 0) {
        TX_CK(cudaMemcpyAsync(tokens, c->otok.p, (size_t) total * 4, cudaMemcpyDeviceToHost, s), "pk_ctc_greedy: copy");
        if (first_frame)
            TX_CK(cudaMemcpyAsync(first_frame, c->oframe.p, (size_t) total * 4, cudaMemcpyDeviceToHost, s),
                  "pk_ctc_greedy: copy");
    }
    TX_CK(cudaMemcpyAsync(prev_inout, c->prev_out.p, (size_t) B * 4, cudaMemcpyDeviceToHost, s), "pk_ctc_greedy: copy");
    TX_CK(cudaStreamSynchronize(s), "pk_ctc_greedy: sync");
    return PK_OK;
}

extern "C" PK_API pk_status pk_vocab_create(int device, const uint8_t * piece_bytes, const int64_t * piece_offsets,
                                            int32_t n_pieces, int32_t blank_id, int32_t bos_id, int32_t eos_id,
                                            int32_t pad_id, pk_vocab ** out) {
    using namespace pk;
    if (!out) return set_error(PK_ERR_INVALID, "pk_vocab_create: null output");
    *out = nullptr;
    if (n_pieces <= 0 || !piece_offsets || (piece_offsets[n_pieces] > 0 && !piece_bytes))
        return set_error(PK_ERR_INVALID, "pk_vocab_create: no pieces");
    for (int v = 0; v < n_pieces; ++v)
        if (piece_offsets[v] < 0 || piece_offsets[v + 1] < piece_offsets[v])
            return set_error(PK_ERR_INVALID, "pk_vocab_create: piece offsets not non-decreasing");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n || !on_sm100(device))
        return set_error(PK_ERR_NO_DEVICE, "pk_vocab_create: no sm_100 device with that index");
    // decoded pieces (sentencepiece_bpe.cpp:15-30): specials empty, each E2 96 81
    // inside a piece one space, every other byte as is
    std::vector<unsigned char> bytes;
    std::vector<int64_t> off((size_t) n_pieces);
    std::vector<int> len((size_t) n_pieces), lead((size_t) n_pieces);
    for (int v = 0; v < n_pieces; ++v) {
        off[v] = (int64_t) bytes.size();
        const bool special = v == blank_id || v == bos_id || v == eos_id || v == pad_id;
        const int64_t a = piece_offsets[v], e = special ? a : piece_offsets[v + 1];
        for (int64_t i = a; i < e;) {
            if (piece_bytes[i] == 0xE2 && i + 2 < e && piece_bytes[i + 1] == 0x96 && piece_bytes[i + 2] == 0x81) {
                bytes.push_back(' ');
                i += 3;
            } else {
                bytes.push_back(piece_bytes[i]);
                ++i;
            }
        }
        len[v] = (int) ((int64_t) bytes.size() - off[v]);
        int ld = 0;
        while (ld < len[v] && bytes[(size_t) off[v] + ld] == ' ') ++ld;
        lead[v] = ld;
    }
    TX_CK(cudaSetDevice(device), "pk_vocab_create: cudaSetDevice");
    pk_vocab * x = new pk_vocab();
    x->device = device;
    x->n = n_pieces;
    auto up = [&](Buf & b, const void * src, size_t nb) -> cudaError_t {
        cudaError_t e = b.ensure(std::max<size_t>(nb, 16));
        if (e == cudaSuccess && nb > 0) e = cudaMemcpy(b.p, src, nb, cudaMemcpyHostToDevice);
        return e;
    };
    cudaError_t e = cudaStreamCreateWithFlags(&x->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = up(x->bytes, bytes.data(), bytes.size());
    if (e == cudaSuccess) e = up(x->off, off.data(), off.size() * 8);
    if (e == cudaSuccess) e = up(x->len, len.data(), len.size() * 4);
    if (e == cudaSuccess) e = up(x->lead, lead.data(), lead.size() * 4);
    if (e != cudaSuccess) {
        pk_vocab_destroy(x);
        return cuda_fail(e, "pk_vocab_create: upload");
    }
    *out = x;
    return PK_OK;
}

extern "C" PK_API void pk_vocab_destroy(pk_vocab * v) {
    if (!v) return;
    cudaSetDevice(v->device);
    if (v->stream) cudaStreamSynchronize(v->stream);
    for (pk::Buf * b : {&v->bytes, &v->off, &v->len, &v->lead, &v->tokens, &v->tokoff, &v->textlen, &v->textlead,
                        &v->textoff, &v->text})
        b->release();
    if (v->stream) cudaStreamDestroy(v->stream);
    delete v;
}

extern "C" PK_API pk_status pk_detokenize(pk_vocab * v, const int32_t * tokens, int32_t tokens_on_device,
                                          const int64_t * token_offsets, int32_t B, char * text, int64_t text_cap,
                                          int64_t * text_offsets, int64_t * text_needed) {
    using namespace pk;
    if (!v || B < 0 || (B > 0 && (!token_offsets || !text_offsets)) || text_cap < 0 || (text_cap > 0 && !text))
        return set_error(PK_ERR_INVALID, "pk_detokenize: null argument or negative size");
    if (B == 0) {
        if (text_offsets) text_offsets[0] = 0;
        if (text_needed) *text_needed = 0;
        return PK_OK;
    }
    if (token_offsets[0] != 0) return set_error(PK_ERR_INVALID, "pk_detokenize: token_offsets[0] must be 0");
    for (int b = 0; b < B; ++b)
        if (token_offsets[b + 1] < token_offsets[b])
            return set_error(PK_ERR_INVALID, "pk_detokenize: token offsets not non-decreasing");
    const int64_t ntok = token_offsets[B];
    if (ntok > 0 && !tokens) return set_error(PK_ERR_INVALID, "pk_detokenize: null tokens");
    if (tokens_on_device && (reinterpret_cast<uintptr_t>(tokens) & 3u))
        return set_error(PK_ERR_INVALID, "pk_detokenize: device tokens must be 4-byte aligned");
    TX_CK(cudaSetDevice(v->device), "pk_detokenize: cudaSetDevice");
    cudaStream_t s = v->stream;
    const int * dtok = tokens;
    if (!tokens_on_device && ntok > 0) {
        TX_CK(v->tokens.ensure((size_t) ntok * 4), "pk_detokenize: alloc");
        TX_CK(cudaMemcpyAsync(v->tokens.p, tokens, (size_t) ntok * 4, cudaMemcpyHostToDevice, s), "pk_detokenize: copy");
        dtok = v->tokens.as<int>();
    }
    TX_CK(v->tokoff.ensure((size_t) (B + 1) * 8), "pk_detokenize: alloc");
    TX_CK(v->textlen.ensure((size_t) B * 4), "pk_detokenize: alloc");
    TX_CK(v->textlead.ensure((size_t) B * 4), "pk_detokenize: alloc");
    TX_CK(v->textoff.ensure((size_t) (B + 1) * 8), "pk_detokenize: alloc");
    TX_CK(cudaMemcpyAsync(v->tokoff.p, token_offsets, (size_t) (B + 1) * 8, cudaMemcpyHostToDevice, s),
          "pk_detokenize: copy");
    VocabDev vd{v->bytes.as<unsigned char>(), v->off.as<int64_t>(), v->len.as<int>(), v->lead.as<int>(), v->n};
    detok_measure_kernel<<<B, kTxtThreads, 0, s>>>(vd, dtok, v->tokoff.as<int64_t>(), v->textlen.as<int>(),
                                                   v->textlead.as<int>());
    TX_CK(cudaGetLastError(), "pk_detokenize: measure launch");
    scan_offsets_kernel<<<1, kTxtThreads, 0, s>>>(v->textlen.as<int>(), B, v->textoff.as<int64_t>());
    TX_CK(cudaGetLastError(), "pk_detokenize: scan launch");
    TX_CK(cudaMemcpyAsync(text_offsets, v->textoff.p, (size_t) (B + 1) * 8, cudaMemcpyDeviceToHost, s),
          "pk_detokenize: offsets copy");
    TX_CK(cudaStreamSynchronize(s), "pk_detokenize: sync");
    const int64_t total = text_offsets[B];
    if (text_needed) *text_needed = total;
    if (total > text_cap) {
        char msg[160];
        std::snprintf(msg, sizeof(msg), "pk_detokenize: %lld bytes > text_cap %lld", (long long) total,
                      (long long) text_cap);
        return set_error(PK_ERR_CAPACITY, msg);
    }
    if (total > 0) {
        TX_CK(v->text.ensure((size_t) total), "pk_detokenize: alloc");
        detok_write_kernel<<<B, kTxtThreads, 0, s>>>(vd, dtok, v->tokoff.as<int64_t>(), v->textlead.as<int>(),
                                                     v->textoff.as<int64_t>(), v->text.as<unsigned char>());
        TX_CK(cudaGetLastError(), "pk_detokenize: write launch");
        TX_CK(cudaMemcpyAsync(text, v->text.p, (size_t) total, cudaMemcpyDeviceToHost, s), "pk_detokenize: copy");
        TX_CK(cudaStreamSynchronize(s), "pk_detokenize: sync");
    }
    return PK_OK;
}
