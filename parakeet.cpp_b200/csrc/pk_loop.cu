// pk_loop.cu -- the persistent greedy-decode step loop (sm_100a).
//
// One cooperative launch (one CTA per SM) runs every step of every utterance
// of a batch. Per batched step:
//
//   [L0 .. L_{L-1}]  LSTM layers for the utterances that emitted (emit list);
//                    CTA k owns hidden units [k*upc, (k+1)*upc) and their four
//                    gate rows (host_lstm_step, src/parakeet_tdt.cpp:106-142)
//   [P]              pred-proj for those utterances, then the joint hidden
//                    hid = relu(enc_proj[t] + pred_proj) for every live one
//                    (host_joint_step, src/parakeet_tdt.cpp:154-177, first half)
//   [J]              joint output rows split over CTAs; per-CTA argmax merged
//                    with 64-bit atomicMax keys (argmax_f32 :25-32: first index
//                    of the maximum wins)
//   leader           the last CTA to reach the barrier applies the greedy
//                    control of tdt_decode_window (:919-969) / eou_decode_window
//                    (parakeet_eou.cpp:267-334) to every live utterance, writes
//                    tokens, and compacts the live and emit lists
//
// Phases are separated by grid barriers whose waits are bounded by a
// globaltimer deadline; a wait that runs out records PK_ERR_TIMEOUT and the
// kernel returns. Cross-CTA data is read with ld.global.cg (L2) after the
// barrier's acquire.
//
// Math here is f32 on CUDA cores with exactly dequantized weights (the
// reference-faithful mode): only the summation order differs from the CPU.

#include "pk_device.cuh"

namespace pk {
namespace {

// Sub-phase timing of CTA 0 in SM clock cycles, compiled in only with
// -DPK_SUBPROF (development builds): SUBMARK(s) adds the cycles since the
// previous mark to slot s (s < 0: restart the interval; -2: publish the slots
// to g_subprof, -3: clear them).
#ifdef PK_SUBPROF
__device__ unsigned long long g_subprof[24];
__device__ __forceinline__ void sub_mark(int slot) {
    __shared__ long long s_t;
    __shared__ unsigned long long s_acc[24];
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        const long long now = clock64();
        if (slot >= 0 && slot < 24) s_acc[slot] += (unsigned long long) (now - s_t);
        if (slot == -2)
            for (int i = 0; i < 24; ++i) g_subprof[i] = s_acc[i];
        if (slot == -3)
            for (int i = 0; i < 24; ++i) s_acc[i] = 0;
        if (slot == -4) s_acc[14] += 1;   // count (leader rounds run by CTA 0)
        s_t = now;
    }
}
#define SUBMARK(s) sub_mark(s)
#else
#define SUBMARK(s) do { } while (0)
#endif

// Shared-memory carve-up of the dynamic buffer.
struct Smem {
    float * xs;                     // [chunk][ldx] activations of one utterance chunk
    float * gates;                  // [chunk][upc][4]
    unsigned long long * wbest;     // [kWarps][32][2]
    int * s_utt;                    // [32]
    int * s_aux;                    // [32] token / step
    int * s_aux2;                   // [32] reset / h-buffer
    int * s_scan;                   // [kWarps + 2]
    int * s_flag;                   // [8]: 0 leader arrival, 1 wait status, 2 staging phase, 4-6 release word
};

__device__ __forceinline__ Smem carve(unsigned char * raw, const LoopParams & P, int upc) {
    Smem s;
    size_t off = 0;
    s.xs = reinterpret_cast<float *>(raw + off);
    off += (size_t) P.chunk * P.ldx * sizeof(float);
    s.gates = reinterpret_cast<float *>(raw + off);
    off += (size_t) P.chunk * upc * 4 * sizeof(float);
    off = (off + 15) & ~(size_t) 15;
    s.wbest = reinterpret_cast<unsigned long long *>(raw + off);
    off += (size_t) kWarps * 32 * 2 * sizeof(unsigned long long);
    s.s_utt = reinterpret_cast<int *>(raw + off); off += 32 * sizeof(int);
    s.s_aux = reinterpret_cast<int *>(raw + off); off += 32 * sizeof(int);
    s.s_aux2 = reinterpret_cast<int *>(raw + off); off += 32 * sizeof(int);
    s.s_scan = reinterpret_cast<int *>(raw + off); off += (kWarps + 2) * sizeof(int);
    s.s_flag = reinterpret_cast<int *>(raw + off);
    return s;
}

// ---- warp dot products over a chunk of CP utterances -----------------------
//
// Lanes split K in float4 slices (k = 4*lane + 128*i); each lane keeps CP
// partial sums, then a butterfly exchange leaves the full sum for utterance
// c = lane >> (5 - log2 CP) in that lane (31 shuffles for CP = 32).
template <int CP>
__device__ __forceinline__ float transpose_reduce(float (&acc)[CP], int lane) {
#pragma unroll
    for (int lev = 0; lev < 5; ++lev) {
        const int o = 16 >> lev;
        const int n = (CP >> lev) > 0 ? (CP >> lev) : 1;
        if (n > 1) {
            const int half = n >> 1;
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < half; ++i) {
                const float send = up ? acc[i] : acc[i + half];
                const float keep = up ? acc[i + half] : acc[i];
                acc[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, o);
            }
        } else {
            acc[0] += __shfl_xor_sync(0xFFFFFFFFu, acc[0], o);
        }
    }
    return acc[0];
}

template <int CP> struct Lg2 {
    static constexpr int v = CP >= 32 ? 5 : CP >= 16 ? 4 : CP >= 8 ? 3 : CP >= 4 ? 2 : CP >= 2 ? 1 : 0;
};

template <int CP>
__device__ __forceinline__ float warp_dot(const float * __restrict__ w, const float * xs, int ldx,
                                          int K, int lane) {
    float acc[CP];
#pragma unroll
    for (int c = 0; c < CP; ++c) acc[c] = 0.0f;
    for (int k = 4 * lane; k < K; k += 128) {
        const float4 wv = __ldg(reinterpret_cast<const float4 *>(w + k));
#pragma unroll
        for (int c = 0; c < CP; ++c) {
            const float4 xv = *reinterpret_cast<const float4 *>(xs + c * ldx + k);
            float a = acc[c];
            a = fmaf(wv.x, xv.x, a);
            a = fmaf(wv.y, xv.y, a);
            a = fmaf(wv.z, xv.z, a);
            a = fmaf(wv.w, xv.w, a);
            acc[c] = a;
        }
    }
    return transpose_reduce<CP>(acc, lane);
}

template <int CP> __device__ __forceinline__ int owner_shift() { return 5 - Lg2<CP>::v; }

__device__ __forceinline__ int pow2ceil(int n) {
    int p = 1;
    while (p < n) p <<= 1;
    return p;
}

__device__ __forceinline__ int lg2_pow2(int p) { return 31 - __clz(p); }

// Stage rows [0, cp) x [0, K) of f32 activations into xs (row stride ldx);
// rows >= nc are zero. Eight independent loads per thread are in flight.
template <class F>
__device__ __forceinline__ void stage_f32(float * xs, int ldx, int cp, int nc, int K, F src) {
    const int k4n = K >> 2;
    const int total = cp * k4n;
    constexpr int U = 8;
    for (int base = 0; base < total; base += U * blockDim.x) {
        float4 vv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int idx = base + u * blockDim.x + threadIdx.x;
            const int c = idx / k4n;
            vv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (idx < total && c < nc) vv[u] = src(c, 4 * (idx - c * k4n));
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int idx = base + u * blockDim.x + threadIdx.x;
            if (idx >= total) break;
            const int c = idx / k4n;
            *reinterpret_cast<float4 *>(xs + c * ldx + 4 * (idx - c * k4n)) = vv[u];
        }
    }
}

// ---- grid barriers -----------------------------------------------------------
//
// Two kinds, on separate words of P.bar (zeroed by the host before each launch):
//  * counter barriers (bar[0]): a monotonically increasing arrival count. Each
//    CTA arrives with one release-ordered reduction (no reply awaited) and waits
//    until the count reaches
//    (k + 1) * gridDim.x for its k-th counter barrier. Nothing is reset, so an
//    arrival costs one reduction and a wait one acquire-load loop.
//  * the leader barrier (bar[2] arrivals, bar[3] generation): the last CTA to
//    arrive runs the control step, resets the arrival word and publishes the
//    next generation with a release store; the others wait for it.

// Returns false if the wait ran out or an error was flagged (thread 0 decides).
template <typename Done>
__device__ __forceinline__ bool bounded_wait(const LoopParams & P, const Smem & S, Done done) {
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned long long t0 = gtimer();
        unsigned it = 0;
        while (!done()) {
            if ((++it & 63u) == 0u) {
                if (__ldcg(&P.ctl[C_ERR]) != 0) { ok = 0; break; }
                if ((long long) (gtimer() - t0) > P.timeout_ns) {
                    atomicCAS(&P.ctl[C_ERR], 0, (int) PK_ERR_TIMEOUT);
                    ok = 0;
                    break;
                }
            }
        }
        S.s_flag[1] = ok;
    }
    __syncthreads();
    return S.s_flag[1] != 0;
}

// k-th counter barrier of this launch (k counts from 0 in every CTA alike).
__device__ __forceinline__ bool grid_barrier(const LoopParams & P, unsigned & k, const Smem & S) {
    __syncthreads();
    const unsigned target = (k + 1u) * gridDim.x;
    if (threadIdx.x == 0) red_add_release(&P.bar[0], 1u);
    ++k;
    return bounded_wait(P, S, [&] { return (int) (ld_acquire(&P.bar[0]) - target) >= 0; });
}

__device__ __forceinline__ bool leader_arrive(const LoopParams & P, const Smem & S) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned old = atom_add_acq_rel(&P.bar[2], 1u);
        S.s_flag[0] = (old == gridDim.x - 1) ? 1 : 0;
        S.s_flag[6] = 0;   // leader: errors seen while deciding
    }
    __syncthreads();
    return S.s_flag[0] != 0;
}

__device__ __forceinline__ unsigned long long * release_word(const LoopParams & P) {
    return reinterpret_cast<unsigned long long *>(P.bar + 4);
}

__device__ __forceinline__ void leader_release(const LoopParams & P, unsigned long long word) {
    __syncthreads();
    if (threadIdx.x == 0) {
        // nobody arrives again before observing the new generation, which the
        // release store orders after this reset and after the CTA's decisions
        // (made visible to thread 0 by the barrier above)
        *reinterpret_cast<volatile unsigned *>(&P.bar[2]) = 0u;
        st_release64(release_word(P), word);
    }
    __syncthreads();
}

// Waits for generation gen + 1; *word receives the release word.
__device__ __forceinline__ bool leader_wait(const LoopParams & P, unsigned gen, const Smem & S,
                                            unsigned long long & word) {
    const unsigned next = (gen + 1u) & 0xFFFFu;
    const bool ok = bounded_wait(P, S, [&] {
        const unsigned long long w = ld_acquire64(release_word(P));
        if ((unsigned) (w >> 48) != next) return false;
        S.s_flag[4] = (int) (unsigned) w;
        S.s_flag[5] = (int) (unsigned) (w >> 32);
        return true;
    });
    word = ((unsigned long long) (unsigned) S.s_flag[5] << 32) | (unsigned) S.s_flag[4];
    return ok;
}

// Block-wide exclusive scan of one int per thread.
__device__ __forceinline__ int block_excl_scan(int v, const Smem & S, int & total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) S.s_scan[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const int w = lane < kWarps ? S.s_scan[lane] : 0;
        int y = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int z = __shfl_up_sync(0xFFFFFFFFu, y, o);
            if (lane >= o) y += z;
        }
        if (lane < kWarps) S.s_scan[lane] = y - w;
        if (lane == kWarps - 1) S.s_scan[kWarps] = y;
    }
    __syncthreads();
    total = S.s_scan[kWarps];
    const int r = x - v + S.s_scan[warp];
    __syncthreads();
    return r;
}

// ---- LSTM layer phase ----------------------------------------------------------

template <int CP>
__device__ void lstm_rows(const LoopParams & P, int l, int u0, int nu, int upc, int nc,
                          const Smem & S) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int H = P.H;
    const int sh = owner_shift<CP>();
    const int c = lane >> sh;
    const bool owner = (lane & ((1 << sh) - 1)) == 0;
    for (int r = warp; r < 4 * nu; r += kWarps) {
        const int jj = r >> 2, q = r & 3;
        const int gr = q * H + u0 + jj;
        const float dih = warp_dot<CP>(P.w_ih[l] + (size_t) gr * H, S.xs, P.ldx, H, lane);
        const float dhh = warp_dot<CP>(P.w_hh[l] + (size_t) gr * H, S.xs + H, P.ldx, H, lane);
        if (owner && c < nc) {
            // g = W_ih x + b_ih; g += b_hh; g += W_hh h  (parakeet_tdt.cpp:123-125)
            const float g = ((__ldg(P.b_ih[l] + gr) + dih) + __ldg(P.b_hh[l] + gr)) + dhh;
            S.gates[(c * upc + jj) * 4 + q] = g;
        }
    }
}

__device__ void phase_lstm(const LoopParams & P, int l, int n_emit, const Smem & S) {
    const int H = P.H, L = P.L, B = P.B;
    const int upc = (H + (int) gridDim.x - 1) / (int) gridDim.x;
    const int u0 = (int) blockIdx.x * upc;
    const int nu = max(0, min(H, u0 + upc) - u0);
    if (nu == 0) return;
    const int K2 = 2 * H;
    for (int cs = 0; cs < n_emit; cs += P.chunk) {
        const int nc = min(P.chunk, n_emit - cs);
        const int cp = pow2ceil(nc);
        if (threadIdx.x < nc) {
            const int utt = __ldcg(&P.emit[2 * (cs + threadIdx.x)]);
            const int tr = __ldcg(&P.emit[2 * (cs + threadIdx.x) + 1]);
            S.s_utt[threadIdx.x] = utt;
            S.s_aux[threadIdx.x] = tr & 0x3FFFFFFF;                              // token
            S.s_aux2[threadIdx.x] = ((tr >> 31) & 1) | (((tr >> 30) & 1) << 1);   // reset | hbuf << 1
        }
        __syncthreads();
        stage_f32(S.xs, P.ldx, cp, nc, K2, [&](int cc, int k) {
            const int utt = S.s_utt[cc];
            const int reset = S.s_aux2[cc] & 1, hb = S.s_aux2[cc] >> 1;
            if (k < H) {
                if (l == 0)
                    return __ldg(reinterpret_cast<const float4 *>(P.embed + (size_t) S.s_aux[cc] * H + k));
                return __ldcg(reinterpret_cast<const float4 *>(P.h + (((size_t) hb * L + (l - 1)) * B + utt) * H + k));
            }
            if (reset) return make_float4(0.f, 0.f, 0.f, 0.f);
            return __ldcg(reinterpret_cast<const float4 *>(P.h + (((size_t) (hb ^ 1) * L + l) * B + utt) * H + (k - H)));
        });
        __syncthreads();
        switch (cp) {
            case 1: lstm_rows<1>(P, l, u0, nu, upc, nc, S); break;
            case 2: lstm_rows<2>(P, l, u0, nu, upc, nc, S); break;
            case 4: lstm_rows<4>(P, l, u0, nu, upc, nc, S); break;
            case 8: lstm_rows<8>(P, l, u0, nu, upc, nc, S); break;
            case 16: lstm_rows<16>(P, l, u0, nu, upc, nc, S); break;
            default: lstm_rows<32>(P, l, u0, nu, upc, nc, S); break;
        }
        __syncthreads();
        // cell update, parakeet_tdt.cpp:128-136
        for (int idx = threadIdx.x; idx < nc * nu; idx += blockDim.x) {
            const int cc = idx / nu, jj = idx - (idx / nu) * nu;
            const int j = u0 + jj;
            const int utt = S.s_utt[cc];
            const int reset = S.s_aux2[cc] & 1, hb = S.s_aux2[cc] >> 1;
            const float * g = S.gates + (cc * upc + jj) * 4;
            const float i_g = sigmoid_ref(g[0]);
            const float f_g = sigmoid_ref(g[1]);
            const float g_g = tanhf(g[2]);
            const float o_g = sigmoid_ref(g[3]);
            float * cptr = P.c + ((size_t) l * B + utt) * H + j;
            const float c_old = reset ? 0.0f : __ldcg(cptr);
            const float c_new = f_g * c_old + i_g * g_g;
            *cptr = c_new;
            P.h[(((size_t) hb * L + l) * B + utt) * H + j] = o_g * tanhf(c_new);
        }
        __syncthreads();
    }
}

// hidden = relu((b_enc + W_enc enc_t) + (b_pred + W_pred pred)) (parakeet_tdt.cpp:168-171)
// for every live utterance and this CTA's joint-hidden rows [j0, j0 + nr). Loads
// are issued four items at a time to keep several L2 requests in flight.
// lutt / lfr: the live list and its encoder rows already in shared memory (the
// whole list), or nullptr to read them from global memory.
__device__ void joint_hidden(const LoopParams & P, int sel, int n_live, int j0, int nr,
                             const int * lutt = nullptr, const long long * lfr = nullptr) {
    const int J = P.J, B = P.B;
    const int * live = lutt ? lutt : P.live + (size_t) sel * B;
    const long long * lframe = lfr ? lfr : reinterpret_cast<const long long *>(P.live_frame) + (size_t) sel * B;
    const int total = n_live * nr;
    for (int base = 0; base < total; base += 4 * blockDim.x) {
        int utt[4], j[4], li[4];
        long long fr[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int idx = base + u * blockDim.x + threadIdx.x;
            utt[u] = -1;
            if (idx < total) {
                const int i = idx / nr;
                li[u] = i;
                j[u] = j0 + (idx - i * nr);
                utt[u] = lutt ? live[i] : __ldcg(&live[i]);
                fr[u] = lfr ? lframe[i] : __ldcg(&lframe[i]);
            }
        }
        float e[4], q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (utt[u] >= 0) {
                e[u] = __ldcg(P.encp + (size_t) fr[u] * J + j[u]);
                q[u] = __ldcg(P.predp + (size_t) utt[u] * J + j[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (utt[u] >= 0) {
                const float v = e[u] + q[u];
                const float hv = (0.0f < v) ? v : 0.0f;
                if (P.tc) {
                    // compact row of live index i in the staged layout: f16 hi | lo
                    const __half hh = __float2half_rn(hv);
                    const __half hl = __float2half_rn(hv - __half2float(hh));
                    __half * row = reinterpret_cast<__half *>(P.hidc + (size_t) li[u] * P.rbj);
                    row[j[u]] = hh;
                    row[J + j[u]] = hl;
                } else {
                    P.hid[(size_t) utt[u] * J + j[u]] = hv;
                }
            }
        }
    }
}

// Trace: LSTM state after the step just decided, for every utterance decided by
// the last leader (the previous live list). Trace mode only (CTA 0).
__device__ void trace_state_dump(const LoopParams & P, bool first, int sel) {
    // (a continued batch's first iteration dumps the bulk loop's last decisions)
    if (P.trace_steps <= 0 || (first && !P.resume) || blockIdx.x != 0) return;
    const int H = P.H, L = P.L, B = P.B;
    const int n_dec = __ldcg(&P.ctl[C_NDECIDED]);
    const int * prev = P.live + (size_t) (sel ^ 1) * B;
    const int LH = L * H;
    for (int i = 0; i < n_dec; ++i) {
        const int utt = __ldcg(&prev[i]);
        const int step = __ldcg(&P.ust[utt * kUst + U_STEPS]) - 1;
        if (step < 0 || step >= P.trace_steps) continue;
        const int hb = __ldcg(&P.ust[utt * kUst + U_HBUF]);
        for (int k = threadIdx.x; k < LH; k += blockDim.x) {
            const int l = k / H, j = k - (k / H) * H;
            const size_t dst = ((size_t) utt * P.trace_steps + step) * LH + k;
            if (P.tr_h) P.tr_h[dst] = __ldcg(P.h + (((size_t) hb * L + l) * B + utt) * H + j);
            if (P.tr_c) P.tr_c[dst] = __ldcg(P.c + ((size_t) l * B + utt) * H + j);
        }
    }
}

// ---- pred-proj + joint hidden phase --------------------------------------------

template <int CP>
__device__ void pred_rows(const LoopParams & P, int j0, int nr, int nc, const Smem & S) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sh = owner_shift<CP>();
    const int c = lane >> sh;
    const bool owner = (lane & ((1 << sh) - 1)) == 0;
    for (int r = warp; r < nr; r += kWarps) {
        const int j = j0 + r;
        const float d = warp_dot<CP>(P.pred_w + (size_t) j * P.H, S.xs, P.ldx, P.H, lane);
        if (owner && c < nc) P.predp[(size_t) S.s_utt[c] * P.J + j] = __ldg(P.pred_b + j) + d;
    }
}

__device__ void phase_pred(const LoopParams & P, bool first, int n_emit, int sel, int n_live,
                           const Smem & S) {
    const int H = P.H, J = P.J, L = P.L, B = P.B;
    const int rpc = (J + (int) gridDim.x - 1) / (int) gridDim.x;
    const int j0 = (int) blockIdx.x * rpc;
    const int nr = max(0, min(J, j0 + rpc) - j0);
    const int * live = P.live + (size_t) sel * B;
    const int n_list = first ? n_live : n_emit;
    if (nr > 0) {
        for (int cs = 0; cs < n_list; cs += P.chunk) {
            const int nc = min(P.chunk, n_list - cs);
            const int cp = pow2ceil(nc);
            if (threadIdx.x < nc) {
                int utt, hb;
                if (first) {
                    utt = __ldcg(&live[cs + threadIdx.x]);
                    hb = __ldcg(&P.ust[utt * kUst + U_HBUF]);
                } else {
                    utt = __ldcg(&P.emit[2 * (cs + threadIdx.x)]);
                    hb = (__ldcg(&P.emit[2 * (cs + threadIdx.x) + 1]) >> 30) & 1;
                }
                S.s_utt[threadIdx.x] = utt;
                S.s_aux2[threadIdx.x] = hb;
            }
            __syncthreads();
            stage_f32(S.xs, P.ldx, cp, nc, H, [&](int cc, int k) {
                return __ldcg(reinterpret_cast<const float4 *>(
                    P.h + (((size_t) S.s_aux2[cc] * L + (L - 1)) * B + S.s_utt[cc]) * H + k));
            });
            __syncthreads();
            switch (cp) {
                case 1: pred_rows<1>(P, j0, nr, nc, S); break;
                case 2: pred_rows<2>(P, j0, nr, nc, S); break;
                case 4: pred_rows<4>(P, j0, nr, nc, S); break;
                case 8: pred_rows<8>(P, j0, nr, nc, S); break;
                case 16: pred_rows<16>(P, j0, nr, nc, S); break;
                default: pred_rows<32>(P, j0, nr, nc, S); break;
            }
            __syncthreads();
        }
        joint_hidden(P, sel, n_live, j0, nr);
        SUBMARK(8);
    }
    trace_state_dump(P, first, sel);
}

// ---- joint output + partial argmax phase ---------------------------------------

template <int CP>
__device__ void joint_rows(const LoopParams & P, int r0, int nr, int nc, const Smem & S,
                           unsigned long long & bt, unsigned long long & bd) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sh = owner_shift<CP>();
    const int c = lane >> sh;
    const bool owner = (lane & ((1 << sh) - 1)) == 0;
    for (int rr = warp; rr < nr; rr += kWarps) {
        const int r = r0 + rr;
        const float d = warp_dot<CP>(P.out_w + (size_t) r * P.J, S.xs, P.ldx, P.J, lane);
        if (owner && c < nc) {
            const float logit = __ldg(P.out_b + r) + d;
            if (P.trace_steps > 0) {
                const int step = S.s_aux[c];
                if (step < P.trace_steps)
                    P.tr_logits[((size_t) S.s_utt[c] * P.trace_steps + step) * P.Vo + r] = logit;
            }
            if (r < P.V1) {
                const unsigned long long k = make_key(logit, r);
                bt = k > bt ? k : bt;
            } else {
                const unsigned long long k = make_key(logit, r - P.V1);
                bd = k > bd ? k : bd;
            }
        }
    }
}

__device__ void phase_joint(const LoopParams & P, int sel, int n_live, const Smem & S, unsigned long long * keys) {
    const int J = P.J, B = P.B;
    const int rpc = (P.Vo + (int) gridDim.x - 1) / (int) gridDim.x;
    const int r0 = (int) blockIdx.x * rpc;
    const int nr = max(0, min(P.Vo, r0 + rpc) - r0);
    if (nr == 0) return;
    const int * live = P.live + (size_t) sel * B;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int cs = 0; cs < n_live; cs += P.chunk) {
        const int nc = min(P.chunk, n_live - cs);
        const int cp = pow2ceil(nc);
        if (threadIdx.x < nc) {
            const int utt = __ldcg(&live[cs + threadIdx.x]);
            S.s_utt[threadIdx.x] = utt;
            S.s_aux[threadIdx.x] = __ldcg(&P.ust[utt * kUst + U_STEPS]);
        }
        __syncthreads();
        stage_f32(S.xs, P.ldx, cp, nc, J, [&](int cc, int k) {
            return __ldcg(reinterpret_cast<const float4 *>(P.hid + (size_t) S.s_utt[cc] * J + k));
        });
        __syncthreads();
        unsigned long long bt = 0ull, bd = 0ull;
        switch (cp) {
            case 1: joint_rows<1>(P, r0, nr, nc, S, bt, bd); break;
            case 2: joint_rows<2>(P, r0, nr, nc, S, bt, bd); break;
            case 4: joint_rows<4>(P, r0, nr, nc, S, bt, bd); break;
            case 8: joint_rows<8>(P, r0, nr, nc, S, bt, bd); break;
            case 16: joint_rows<16>(P, r0, nr, nc, S, bt, bd); break;
            default: joint_rows<32>(P, r0, nr, nc, S, bt, bd); break;
        }
        // lanes that own utterance c hold the warp's best keys; gather per warp
        const int sh = 5 - lg2_pow2(cp);
        if ((lane & ((1 << sh) - 1)) == 0) {
            const int c = lane >> sh;
            S.wbest[(warp * 32 + c) * 2 + 0] = bt;
            S.wbest[(warp * 32 + c) * 2 + 1] = bd;
        }
        __syncthreads();
        if (threadIdx.x < nc) {
            unsigned long long kt = 0ull, kd = 0ull;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const unsigned long long a = S.wbest[(w * 32 + threadIdx.x) * 2 + 0];
                const unsigned long long b = S.wbest[(w * 32 + threadIdx.x) * 2 + 1];
                kt = a > kt ? a : kt;
                kd = b > kd ? b : kd;
            }
            const int utt = S.s_utt[threadIdx.x];
            if (kt) atomicMax(&keys[2 * utt + 0], kt);
            if (kd) atomicMax(&keys[2 * utt + 1], kd);
        }
        __syncthreads();
    }
}

// ---- leader: greedy control for every live utterance -------------------------

// The last CTA to reach the joint barrier decides every live utterance's step:
// argmax keys -> token / duration, frame advance, token output, and the next
// iteration's live and emit lists (compacted with one block scan). sel / n_live
// are the current list selector and length; every CTA read them at the start of
// the iteration and nothing has changed them since.
// live_smem: the whole live list already in shared memory, or nullptr.
// keys: this iteration's argmax key buffer (cleared here for its next use).
__device__ unsigned long long leader_decide(const LoopParams & P, const Smem & S, int sel, int n_live,
                                           unsigned gen_next, unsigned long long * keys,
                                           const int * live_smem = nullptr) {
    const int B = P.B;
    // an error flagged anywhere so far travels with the release word
    const int err0 = threadIdx.x == 0 ? __ldcg(&P.ctl[C_ERR]) : 0;
    const int * live_in = P.live + (size_t) sel * B;
    int * live_out = P.live + (size_t) (sel ^ 1) * B;
    int base_emit = 0, base_live = 0;
    for (int r0 = 0; r0 < n_live; r0 += blockDim.x) {
        const int i = r0 + threadIdx.x;
        int e = 0, lv = 0, utt = -1, etok = 0, ereset = 0, ehb = 0;
        long long lframe = 0;
        if (i < n_live) {
            utt = live_smem ? live_smem[i] : __ldcg(&live_in[i]);
            int * u = P.ust + utt * kUst;
            // every load that depends only on utt goes out together (one round trip)
            const unsigned long long kt = __ldcg(&keys[2 * utt + 0]);
            const unsigned long long kd = P.is_tdt ? __ldcg(&keys[2 * utt + 1]) : 0ull;
            const int4 u0 = __ldcg(reinterpret_cast<const int4 *>(u));
            const int4 u1 = __ldcg(reinterpret_cast<const int4 *>(u) + 1);
            const int4 u2 = __ldcg(reinterpret_cast<const int4 *>(u) + 2);
            const long long foff = __ldg(P.frame_off + utt);
            int uf[12] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w, u2.x, u2.y, u2.z, u2.w};
            // the next joint phase on this buffer max-reduces into cleared keys
            // (ordered by the barrier release)
            keys[2 * utt + 0] = 0ull;
            if (P.is_tdt) keys[2 * utt + 1] = 0ull;
            int tok = key_index(kt);
            int di = P.is_tdt ? key_index(kd) : 0;
            if (keys_bad(P, kt, kd, tok, di)) {
                atomicCAS(&P.ctl[C_ERR], 0, (int) PK_ERR_DEVICE);
                atomicOr(&S.s_flag[6], 1);
                P.ctl[C_ERRINFO] = utt;
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
            const int sym = d.sym;
            e = d.e; etok = d.etok; ereset = d.ereset;
            int ntok = uf[U_NTOK];
            if (!P.is_tdt) eou_effects(P, u, uf, utt, d, s0, ntok, tok, T);
            if (d.emit_tok) {
                if (!put_token(P, utt, tok, ntok, T)) atomicOr(&S.s_flag[6], 1);
            }
            if (e) {
                ehb = uf[U_HBUF] ^ 1;
                u[U_HBUF] = ehb;
            }
            u[U_T] = t;
            u[U_SYM] = sym;
            u[U_NTOK] = ntok;
            lv = t < T ? 1 : 0;
            if (lv) lframe = foff + t;
            if (!lv) P.finish_ns[utt] = gtimer();
        }
        // one scan for both lists: emit count in the low half, live count in the high half
        int tot = 0;
        const int pf = block_excl_scan(e | (lv << 16), S, tot);
        const int pe = pf & 0xFFFF, pl = pf >> 16;
        if (e) {
            reinterpret_cast<int2 *>(P.emit)[base_emit + pe] = make_int2(utt, etok | (ehb << 30) | (ereset << 31));
        }
        if (lv) {
            live_out[base_live + pl] = utt;
            P.live_frame[(size_t) (sel ^ 1) * B + base_live + pl] = lframe;
        }
        base_emit += tot & 0xFFFF;
        base_live += tot >> 16;
    }
    if (threadIdx.x == 0) {
        P.ctl[C_NEMIT] = base_emit;
        P.ctl[C_NLIVE0 + (sel ^ 1)] = base_live;
        P.ctl[C_NDECIDED] = n_live;
        P.ctl[C_SEL] = sel ^ 1;
        if (err0 != 0) atomicOr(&S.s_flag[6], 1);
    }
    __syncthreads();
    const int err = S.s_flag[6];
    return pack_ctl(gen_next, err, sel ^ 1, base_emit, base_live);
}

// ---- tensor-core phases (PK_MATH_TC) -------------------------------------------
//
// Each phase is a small GEMM C[rows of this CTA][16 utterances] = W . X^T on the
// warp-level tensor cores, 16 utterances (one pass) at a time, the 8 warps
// splitting K in 32-wide blocks with a shared-memory reduction. Weights are
// exact. Activations keep f32-level accuracy:
//  * h (LSTM outputs, |h| < 1) with q8_0 weights: int16 fixed point h * 2^15 as
//    two int8 digits (hi signed, lo unsigned); mma.m16n8k32 s8 / u8 x s8 gives
//    each 32-wide q8_0 block's exact int32 product, scaled by the block's d.
//  * otherwise (hid, or f16 weights): f16 hi + lo halves (x = hi + lo to 22
//    significant bits), two mma.m16n8k16 per weight fragment; q8_0 weights enter
//    as exact f16 integers with the block scale applied per 32-wide block.
//
// Activation rows live in HBM in the layout they take in shared memory: the hi
// part, then the lo part, padded to a row stride (rbh for h, rbj for hid) of
// 16 mod 128 bytes so that ldmatrix rows hit distinct banks. Producers write
// them twice where a consumer reads a whole pass: the LSTM cell update writes
// each new h both to the utterance's state row and to a compact row indexed by
// its position in the emit list, and the joint hidden layer is written by
// position in the live list, so the next phase stages a pass with a single
// bulk copy. Only rows indexed by utterance (h_prev, read back at the
// utterance's next emission) are copied row by row.

struct TcSmem {
    unsigned char * w;              // stationary weights (P.sm_weights bytes)
    unsigned char * area;           // staging area (P.area bytes): the pass's activation rows, then the
                                    // GEMM's per-warp partial sums once the rows have been read
    float * C;                      // [kTcRmax][8][16 * mb] reduced GEMM output
    unsigned long long * mbar;      // staging completion barrier (bulk copies)
    int * s_utt;                    // [kTcRec] records of the current block
    int * s_aux;                    // [kTcRec]
    int * s_aux2;                   // [kTcRec]
    int * s_lutt;                   // [kTcRec] first block of the live list (loaded with the emit records)
    long long * s_lframe;           // [kTcRec] its encoder rows
    int2 * s_lst;                   // [kTcRec] its control state in replicated mode:
                                    // (frames left, symbol count | h buffer << 30)
    int * s_scan;                   // [kWarps + 2]
    int * s_flag;                   // [8]: 0 leader arrival, 1 wait status, 2 staging phase, 4-6 release word
    float * bj;                     // [rpc_j] this CTA's joint-out bias slice
    float * bp;                     // [rpc_p] this CTA's pred-proj bias slice
    float * lb;                     // [L][4][upc] LSTM gate biases of this CTA's units
};

__device__ __forceinline__ TcSmem tc_carve(unsigned char * raw, const LoopParams & P) {
    TcSmem s;
    size_t off = 0;
    s.w = raw;
    off += (P.sm_weights + 15) & ~15u;
    s.area = raw + off; off += (size_t) P.area;
    s.C = reinterpret_cast<float *>(raw + off); off += (size_t) kTcRmax * 128 * 2 * 4;
    s.mbar = reinterpret_cast<unsigned long long *>(raw + off); off += 16;
    s.s_utt = reinterpret_cast<int *>(raw + off); off += kTcRec * 4;
    s.s_aux = reinterpret_cast<int *>(raw + off); off += kTcRec * 4;
    s.s_aux2 = reinterpret_cast<int *>(raw + off); off += kTcRec * 4;
    s.s_lutt = reinterpret_cast<int *>(raw + off); off += kTcRec * 4;
    s.s_lframe = reinterpret_cast<long long *>(raw + off); off += kTcRec * 8;
    s.s_lst = reinterpret_cast<int2 *>(raw + off); off += kTcRec * 8;
    s.s_scan = reinterpret_cast<int *>(raw + off); off += (kWarps + 2) * 4;
    s.s_flag = reinterpret_cast<int *>(raw + off); off += 8 * 4;
    s.bj = reinterpret_cast<float *>(raw + off); off += (size_t) P.rpc_j * 4;
    s.bp = reinterpret_cast<float *>(raw + off); off += (size_t) P.rpc_p * 4;
    s.lb = reinterpret_cast<float *>(raw + off);
    return s;
}

// The barrier / scan helpers only use s_scan and s_flag.
__device__ __forceinline__ TcSmem tc_pass(const TcSmem & T, int p) {
    TcSmem q = T;
    q.s_utt += p; q.s_aux += p; q.s_aux2 += p;
    return q;
}

__device__ __forceinline__ Smem as_smem(const TcSmem & T) {
    Smem s{};
    s.s_utt = T.s_utt; s.s_aux = T.s_aux; s.s_aux2 = T.s_aux2; s.s_scan = T.s_scan; s.s_flag = T.s_flag;
    return s;
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const unsigned char * p) {
    const unsigned a = (unsigned) __cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a) : "memory");
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    // no side effects beyond its registers: left free for the scheduler
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// int8 tensor-core products (exact int32): A digit plane x raw q8_0 bytes.
__device__ __forceinline__ void imma_s8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void imma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Four biased bytes (q + 128) -> two f16x2 holding q exactly: byte b placed
// under the f16 exponent of 1024 gives 1024 + b, minus 1152 gives q.
__device__ __forceinline__ void biased_i8x4_to_h2x2(uint32_t v, uint32_t & lo, uint32_t & hi) {
    const uint32_t a = __byte_perm(v, 0x64646464u, 0x4140);
    const uint32_t b = __byte_perm(v, 0x64646464u, 0x4342);
    const __half2 bias = __half2half2(__ushort_as_half((unsigned short) 0x6480));  // 1152
    __half2 ha = __hsub2(*reinterpret_cast<const __half2 *>(&a), bias);
    __half2 hb = __hsub2(*reinterpret_cast<const __half2 *>(&b), bias);
    lo = *reinterpret_cast<uint32_t *>(&ha);
    hi = *reinterpret_cast<uint32_t *>(&hb);
}

// Stage one pass (rows [0, nc), nc <= 16 * mb) with bulk copies (the copy
// engine), completion counted on S.mbar:
//  * tile (optional): nc contiguous rows of tile_rb bytes to dtile, one slice per warp;
//  * per-row (drows != nullptr): drows + c * rows_rb <- row_bytes bytes at
//    rowsrc(c), or zeros where rowsrc(c) is nullptr.
// Lane 0 of every warp issues its share of the copies and arrives once with its
// byte count. Rows nc..15 keep whatever they held: each mma output row depends
// on its own A row only, and outputs of rows >= nc are never read. Generic-proxy
// accesses of the regions (ldmatrix reads in tc_gemm_nt, the zero stores here
// and at kernel start) are each followed by fence.proxy.async in the thread that
// made them and by a CTA barrier before the next stage issues its copies.
// Returns false (error flagged) if the copies did not complete within timeout_ns.
template <typename F>
__device__ __forceinline__ bool tc_stage(const LoopParams & P, const TcSmem & S, int nc,
                                         const unsigned char * tile, unsigned tile_rb, unsigned char * dtile,
                                         unsigned char * drows, unsigned row_bytes, unsigned rows_rb, F rowsrc) {
    SUBMARK(17);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned ph = (unsigned) S.s_flag[2];
    const unsigned mb = (unsigned) __cvta_generic_to_shared(S.mbar);
    if (drows != nullptr) {
        for (int c = warp; c < nc; c += kWarps) {
            if (rowsrc(c) == nullptr) {
                unsigned char * d = drows + (size_t) c * rows_rb;
                for (unsigned k = lane * 16u; k < row_bytes; k += 32u * 16u)
                    *reinterpret_cast<uint4 *>(d + k) = make_uint4(0u, 0u, 0u, 0u);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            }
        }
    }
    if (lane == 0) {
        // the tile goes in one 16-byte-aligned slice per warp: one issuing
        // thread reaches about half the shared-memory fill rate that eight do
        const unsigned ttot = tile != nullptr ? (unsigned) nc * tile_rb : 0u;
        const unsigned tchunk = ((ttot / kWarps) + 15u) & ~15u;
        const unsigned tbeg = min(ttot, (unsigned) warp * tchunk), tlen = min(ttot, tbeg + tchunk) - tbeg;
        unsigned mine = tlen;
        if (drows != nullptr)
            for (int c = warp; c < nc; c += kWarps)
                if (rowsrc(c) != nullptr) mine += row_bytes;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(mb), "r"(mine) : "memory");
        if (tlen > 0u) {
            const unsigned da = (unsigned) __cvta_generic_to_shared(dtile + tbeg);
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                         :: "r"(da), "l"(tile + tbeg), "r"(tlen), "r"(mb) : "memory");
        }
        if (drows != nullptr) {
            for (int c = warp; c < nc; c += kWarps) {
                const unsigned char * g = rowsrc(c);
                if (g == nullptr) continue;
                const unsigned da = (unsigned) __cvta_generic_to_shared(drows + (size_t) c * rows_rb);
                asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                             :: "r"(da), "l"(g), "r"(row_bytes), "r"(mb) : "memory");
            }
        }
    }
    SUBMARK(15);
    // every thread waits for the phase itself (the completed wait orders the copied
    // data for it), each with the same bound; one barrier agrees on the outcome
    int fail = 0;
    {
        const unsigned long long t0 = gtimer();
        for (unsigned it = 1;; ++it) {
            unsigned done;
            asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                         : "=r"(done) : "r"(mb), "r"(ph) : "memory");
            if (done) break;
            if ((it & 63u) == 0u && (long long) (gtimer() - t0) > P.timeout_ns) { fail = 1; break; }
        }
    }
    const bool ok = __syncthreads_or(fail) == 0;   // everyone has read the phase bit before it flips
    SUBMARK(16);
    if (threadIdx.x == 0) {
        if (!ok) atomicCAS(&P.ctl[C_ERR], 0, (int) PK_ERR_TIMEOUT);
        S.s_flag[2] = (int) (ph ^ 1u);
    }
    return ok;
}

// PK_MATH_Q8: the staged activation rows [0, nc) at base (stride rb) become q8_0
// blocks in place, as ggml's quantize_row_q8_0 makes them for vec_dot_q8_0_q8_0:
// per 32 consecutive values d = max|x| / 127, q = roundf(x / d) (0 when d = 0), d
// kept as binary16. K values per row, read as int16 fixed point (two int8 digit
// planes, hi at +k, lo at +lo + k: x = (hi * 256 + lo) / 2^15) or as f16 halves
// (hi at +2k, lo at +lo + 2k: x = hi + lo). Written: q at byte positions [0, K),
// in the k order of the B fragments the GEMM pairs them with (identity for
// mma.m16n8k32 fragments; the k16-fragment order of the joint's weights when
// perm), and d (f32 of its binary16 value) at +lo + 4 * block. One warp per row,
// lane l holding value 32 b + l of block b: every lane has read a block (before
// the block's max reduction) before any lane writes it, and a block's writes only
// touch bytes of values of that block or of earlier ones.
__device__ void q8_rows(unsigned char * base, int nc, int rb, int K, int lo, bool src_i16, bool perm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // position of value kk (< 16) of a k16 half within the fragment order: lane t of
    // the k16 fragments holds kk = 2t, 2t + 1, 2t + 8, 2t + 9 at positions 4t .. 4t + 3
    const int kk = lane & 15;
    const int pos = perm ? ((lane & 16) + 4 * ((kk & 7) >> 1) + (kk & 1) + 2 * (kk >> 3)) : lane;
    for (int c = warp; c < nc; c += kWarps) {
        unsigned char * row = base + (size_t) c * rb;
        for (int b = 0; b < (K >> 5); ++b) {
            const int k = 32 * b + lane;
            float x;
            if (src_i16) {
                x = (float) ((int) (signed char) row[k] * 256 + (int) row[lo + k]) * (1.0f / 32768.0f);
            } else {
                x = __half2float(reinterpret_cast<const __half *>(row)[k]) +
                    __half2float(reinterpret_cast<const __half *>(row + lo)[k]);
            }
            float amax = fabsf(x);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
            const float d = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            const int q = (int) roundf(x * id);
            row[32 * b + pos] = (unsigned char) (signed char) q;
            if (lane == 0) *reinterpret_cast<float *>(row + lo + 4 * b) = __half2float(__float2half_rn(d));
            __syncwarp();
        }
    }
    __syncthreads();
}

__device__ __forceinline__ const uint8_t * tc_frag(const LoopParams & P, const TcSmem & S, const TcBlock & b) {
    return P.stationary ? S.w + b.sm_frag : b.frag + (size_t) blockIdx.x * b.cta_bytes;
}
__device__ __forceinline__ const float * tc_scale(const LoopParams & P, const TcSmem & S, const TcBlock & b) {
    return P.stationary ? reinterpret_cast<const float *>(S.w + b.sm_scale)
                        : b.scale + (size_t) blockIdx.x * b.cta_scales;
}

// Where the staged A of a GEMM lives: K blocks below kb_split in the rows at
// r0, the rest in the rows at r1 (row stride rb bytes; lo part lo bytes into a
// row). m16 block m of the pass starts 16 * m rows further on.
struct ATile {
    const unsigned char * r0;
    const unsigned char * r1;
    int rb, lo, kb_split;
};

// C[r][col][c] (r < NT tiles starting at tile t0, col = row within the tile,
// c < 16 * MB = utterance of the pass) for the staged activations. Each warp
// takes a 1/8 slice of the K blocks for all NT tiles and MB m16 blocks (the
// weight fragments are loaded once for the MB blocks); the slices are summed
// through shared memory, in the staging area, whose rows are no longer needed
// once every warp has finished its ldmatrix reads. NT and MB are compile-time
// constants so the per-tile work carries no predicates.
// kw (4 or 8): warps that split K. Fewer warps halve the partial sums to
// reduce; the tensor pipe stays busy with one warp per scheduler for the
// joint's many tiles and for passes of one m16 block.
// keep: bytes of activation rows at the start of the staging area. When the
// partial sums fit after them they go to the end of the area, the rows survive
// the call (a phase's next call on further tiles reads them again) and no CTA
// barrier has to separate the warps' last row reads from the partial writes.
template <int NT, int MB, bool Q8>
__device__ void tc_gemm_nt(const LoopParams & P, const TcSmem & S, const TcBlock & b, int t0, const ATile & A,
                           int kw, int keep) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t = lane & 3, g = lane >> 2;
    const int nkb = b.K >> 5;
    const int kb0 = warp < kw ? (warp * nkb) / kw : 0, kb1 = warp < kw ? ((warp + 1) * nkb) / kw : 0;
    const uint8_t * frag = tc_frag(P, S, b);
    const float * scale = tc_scale(P, S, b);
    float acc[NT][MB][4];
#pragma unroll
    for (int r = 0; r < NT; ++r)
#pragma unroll
        for (int m = 0; m < MB; ++m) acc[r][m][0] = acc[r][m][1] = acc[r][m][2] = acc[r][m][3] = 0.0f;
    const int mrow = ((lane >> 3) & 1) * 8 + (lane & 7);
    const int mb16 = (lane >> 4) * 16;                 // byte column of this lane's ldmatrix row
    const int kbytes = (b.imma || Q8) ? 32 : 64;       // bytes of one 32-wide K block per part
    const size_t mstep = (size_t) 16 * A.rb;           // bytes between m16 blocks
    const unsigned char * a0 = A.r0 + mrow * A.rb + mb16;
    const unsigned char * a1 = A.r1 + mrow * A.rb + mb16 - A.kb_split * kbytes;
    if constexpr (Q8) {
        // q8_0 activations (q8_rows) x q8_0 weights: one int8 product per block, scaled
        // by the weight row's d and the activation row's d (vec_dot_q8_0_q8_0)
        const uint32_t flip = b.imma ? 0u : 0x80808080u;   // biased bytes q + 128 -> int8 q
        for (int kb = kb0; kb < kb1; ++kb) {
            const bool first = kb < A.kb_split;
            const unsigned char * hp = (first ? a0 : a1) + kb * 32;
            const unsigned char * dp = (first ? A.r0 : A.r1) + g * A.rb + A.lo + 4 * (first ? kb : kb - A.kb_split);
            uint32_t aq[MB][4];
            float dx0[MB], dx1[MB];
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                ldsm_x4(aq[m], hp + m * mstep);
                dx0[m] = *reinterpret_cast<const float *>(dp + m * mstep);
                dx1[m] = *reinterpret_cast<const float *>(dp + m * mstep + 8 * A.rb);
            }
#pragma unroll
            for (int r = 0; r < NT; ++r) {
                const size_t u = (size_t) (t0 + r) * nkb + kb;
                const uint2 w = *reinterpret_cast<const uint2 *>(frag + (u * 32 + lane) * 8);
                const float2 sc = *reinterpret_cast<const float2 *>(scale + u * 8 + 2 * t);
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    int dq[4] = {0, 0, 0, 0};
                    imma_s8s8(dq, aq[m], w.x ^ flip, w.y ^ flip);
                    acc[r][m][0] = fmaf(sc.x * dx0[m], (float) dq[0], acc[r][m][0]);
                    acc[r][m][1] = fmaf(sc.y * dx0[m], (float) dq[1], acc[r][m][1]);
                    acc[r][m][2] = fmaf(sc.x * dx1[m], (float) dq[2], acc[r][m][2]);
                    acc[r][m][3] = fmaf(sc.y * dx1[m], (float) dq[3], acc[r][m][3]);
                }
            }
        }
    } else {
    if (b.imma) {
        for (int kb = kb0; kb < kb1; ++kb) {
            const unsigned char * hp = (kb < A.kb_split ? a0 : a1) + kb * 32;
            uint32_t ah[MB][4], al[MB][4];
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                ldsm_x4(ah[m], hp + m * mstep);
                ldsm_x4(al[m], hp + m * mstep + A.lo);
            }
#pragma unroll
            for (int r = 0; r < NT; ++r) {
                const size_t u = (size_t) (t0 + r) * nkb + kb;
                const uint2 w = *reinterpret_cast<const uint2 *>(frag + (u * 32 + lane) * 8);
                const float2 sc = *reinterpret_cast<const float2 *>(scale + u * 8 + 2 * t);
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    int dh[4] = {0, 0, 0, 0}, dl[4] = {0, 0, 0, 0};
                    imma_s8s8(dh, ah[m], w.x, w.y);
                    imma_u8s8(dl, al[m], w.x, w.y);
                    acc[r][m][0] = fmaf(sc.x, (float) (dh[0] * 256 + dl[0]), acc[r][m][0]);
                    acc[r][m][1] = fmaf(sc.y, (float) (dh[1] * 256 + dl[1]), acc[r][m][1]);
                    acc[r][m][2] = fmaf(sc.x, (float) (dh[2] * 256 + dl[2]), acc[r][m][2]);
                    acc[r][m][3] = fmaf(sc.y, (float) (dh[3] * 256 + dl[3]), acc[r][m][3]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < NT; ++r)
#pragma unroll
            for (int m = 0; m < MB; ++m)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[r][m][q] *= 1.0f / 32768.0f;
    } else if (b.is_i8) {
        for (int kb = kb0; kb < kb1; ++kb) {
            const unsigned char * hp = (kb < A.kb_split ? a0 : a1) + kb * 64;
            uint32_t ah0[MB][4], al0[MB][4], ah1[MB][4], al1[MB][4];
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                ldsm_x4(ah0[m], hp + m * mstep);
                ldsm_x4(al0[m], hp + m * mstep + A.lo);
                ldsm_x4(ah1[m], hp + m * mstep + 32);
                ldsm_x4(al1[m], hp + m * mstep + A.lo + 32);
            }
#pragma unroll
            for (int r = 0; r < NT; ++r) {
                const size_t u = (size_t) (t0 + r) * nkb + kb;
                const uint2 w = *reinterpret_cast<const uint2 *>(frag + (u * 32 + lane) * 8);
                const float2 sc = *reinterpret_cast<const float2 *>(scale + u * 8 + 2 * t);
                uint32_t b0, b1, b2, b3;
                biased_i8x4_to_h2x2(w.x, b0, b1);
                biased_i8x4_to_h2x2(w.y, b2, b3);
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    // one chain over the block's hi and lo parts (two k16 steps
                    // each); the q8_0 block scale is applied to the sum
                    float th[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(th, ah0[m], b0, b1);
                    mma16816(th, al0[m], b0, b1);
                    mma16816(th, ah1[m], b2, b3);
                    mma16816(th, al1[m], b2, b3);
                    acc[r][m][0] = fmaf(sc.x, th[0], acc[r][m][0]);
                    acc[r][m][1] = fmaf(sc.y, th[1], acc[r][m][1]);
                    acc[r][m][2] = fmaf(sc.x, th[2], acc[r][m][2]);
                    acc[r][m][3] = fmaf(sc.y, th[3], acc[r][m][3]);
                }
            }
        }
    } else {
        for (int kb = kb0; kb < kb1; ++kb) {
            const unsigned char * hp = (kb < A.kb_split ? a0 : a1) + kb * 64;
            uint32_t ah0[MB][4], al0[MB][4], ah1[MB][4], al1[MB][4];
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                ldsm_x4(ah0[m], hp + m * mstep);
                ldsm_x4(al0[m], hp + m * mstep + A.lo);
                ldsm_x4(ah1[m], hp + m * mstep + 32);
                ldsm_x4(al1[m], hp + m * mstep + A.lo + 32);
            }
#pragma unroll
            for (int r = 0; r < NT; ++r) {
                const size_t u = (size_t) (t0 + r) * nkb + kb;
                const uint4 w = *reinterpret_cast<const uint4 *>(frag + (u * 32 + lane) * 16);
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    mma16816(acc[r][m], ah0[m], w.x, w.y);
                    mma16816(acc[r][m], al0[m], w.x, w.y);
                    mma16816(acc[r][m], ah1[m], w.z, w.w);
                    mma16816(acc[r][m], al1[m], w.z, w.w);
                }
            }
        }
    }
    }
    constexpr int W = 16 * MB;                         // utterance columns of a partial tile
    // rows padded to W + 4 floats: a store's 32 lanes (rows 2t / 2t + 1, columns g)
    // then fall on 32 distinct banks (2 (W + 4) = 8 mod 32)
    constexpr int WP = W + 4;
    const int end_off = (P.area - kw * NT * 8 * WP * 4) & ~15;
    const bool at_end = keep > 0 && end_off >= keep;
    // otherwise every warp's ldmatrix reads are done before the partial sums overwrite the rows
    if (!at_end) __syncthreads();
    float * part = reinterpret_cast<float *>(S.area + (at_end ? end_off : 0));  // [kw][NT][8][WP]
    if (warp < kw) {
#pragma unroll
        for (int r = 0; r < NT; ++r) {
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                float * pp = part + ((warp * NT + r) * 8) * WP + m * 16;
                pp[(2 * t) * WP + g] = acc[r][m][0];
                pp[(2 * t + 1) * WP + g] = acc[r][m][1];
                pp[(2 * t) * WP + g + 8] = acc[r][m][2];
                pp[(2 * t + 1) * WP + g + 8] = acc[r][m][3];
            }
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < NT * 8 * W; idx += blockDim.x) {
        const int pi = (idx / W) * WP + idx % W;
        float s = 0.0f;
        for (int w = 0; w < kw; ++w) s += part[w * NT * 8 * WP + pi];
        S.C[idx] = s;
    }
    // this thread's generic accesses of the area come before the next stage's bulk writes
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
}

// C layout: row r of the pass's tile group, utterance c -> C[(r >> 3) * 8 * W + (r & 7) * W + c].
__device__ __forceinline__ int c_index(int r, int c, int W) { return (r >> 3) * 8 * W + (r & 7) * W + c; }

// mbp: m16 blocks of this pass (2 only when the pass has more than 16
// utterances and the loop was set up for 32-utterance passes). Two-block calls
// take at most 7 tiles, one-block calls 8 (callers split larger groups).
template <bool Q8>
__device__ __forceinline__ void tc_gemm_q(const LoopParams & P, const TcSmem & S, const TcBlock & b, int t0, int nt,
                                        const ATile & A, int mbp, int kw, int keep = 0) {
    if (mbp == 2) {
        switch (nt) {
            case 1: tc_gemm_nt<1, 2, Q8>(P, S, b, t0, A, kw, keep); break;
            case 2: tc_gemm_nt<2, 2, Q8>(P, S, b, t0, A, kw, keep); break;
            case 3: tc_gemm_nt<3, 2, Q8>(P, S, b, t0, A, kw, keep); break;
            case 4: tc_gemm_nt<4, 2, Q8>(P, S, b, t0, A, kw, keep); break;
            case 5: tc_gemm_nt<5, 2, Q8>(P, S, b, t0, A, kw, keep); break;
            case 6: tc_gemm_nt<6, 2, Q8>(P, S, b, t0, A, kw, keep); break;
            default: tc_gemm_nt<7, 2, Q8>(P, S, b, t0, A, kw, keep); break;
        }
        return;
    }
    switch (nt) {
        case 1: tc_gemm_nt<1, 1, Q8>(P, S, b, t0, A, kw, keep); break;
        case 2: tc_gemm_nt<2, 1, Q8>(P, S, b, t0, A, kw, keep); break;
        case 3: tc_gemm_nt<3, 1, Q8>(P, S, b, t0, A, kw, keep); break;
        case 4: tc_gemm_nt<4, 1, Q8>(P, S, b, t0, A, kw, keep); break;
        case 5: tc_gemm_nt<5, 1, Q8>(P, S, b, t0, A, kw, keep); break;
        case 6: tc_gemm_nt<6, 1, Q8>(P, S, b, t0, A, kw, keep); break;
        case 7: tc_gemm_nt<7, 1, Q8>(P, S, b, t0, A, kw, keep); break;
        default: tc_gemm_nt<8, 1, Q8>(P, S, b, t0, A, kw, keep); break;
    }
}


// Records of one emit-list block: utterance, token, reset | h buffer << 1.
__device__ __forceinline__ void tc_emit_record(const LoopParams & P, const TcSmem & T, int i, int g) {
    const int2 e = __ldcg(reinterpret_cast<const int2 *>(P.emit) + g);
    T.s_utt[i] = e.x;
    T.s_aux[i] = e.y & 0x3FFFFFFF;
    T.s_aux2[i] = ((e.y >> 31) & 1) | (((e.y >> 30) & 1) << 1);
}

// The joint-hidden step reads each live utterance's enc-proj row after the
// LSTM phases: pull the rows of the live entries in shared memory into L2 at
// the start of the iteration (one bulk prefetch per row, spread over the CTAs),
// since the enc-proj table of a long batch exceeds L2.
__device__ __forceinline__ void tc_prefetch_encp(const LoopParams & P, const TcSmem & T, int nl) {
    for (int i = (int) blockIdx.x + (int) threadIdx.x * (int) gridDim.x; i < nl; i += (int) (blockDim.x * gridDim.x))
        prefetch_l2(P.encp + (size_t) T.s_lframe[i] * P.J, (unsigned) P.J * 4u);
}

// Iterations whose live list fits shared memory end with a decision that every
// CTA computes itself (no leader round trip); trace runs keep the leader.
__device__ __forceinline__ bool rep_mode(const LoopParams & P, int n_live) {
    return P.trace_steps <= 0 && n_live <= kTcRec;
}

// Start of an iteration: the first block of the emit list (LSTM and pred-proj
// records) and of the live list (joint records) in one round trip. When a list
// fits one block the phases use these copies instead of reloading.
__device__ __forceinline__ void tc_load_records(const LoopParams & P, const TcSmem & T, int sel, int n_emit,
                                                int n_live) {
    const int ne = min(kTcRec, n_emit), nl = min(kTcRec, n_live);
    const int * live = P.live + (size_t) sel * P.B;
    // the iteration ends with a replicated decision: each CTA takes its own copy
    // of the live utterances' control state (kept in shared memory from then on)
    const bool rep = rep_mode(P, n_live);
    for (int i = threadIdx.x; i < max(ne, nl); i += blockDim.x) {
        if (i < ne) tc_emit_record(P, T, i, i);
        if (i < nl) {
            const int utt = __ldcg(&live[i]);
            T.s_lutt[i] = utt;
            T.s_lframe[i] = __ldcg(reinterpret_cast<const long long *>(P.live_frame) + (size_t) sel * P.B + i);
            if (rep) {
                const int * u = P.ust + utt * kUst;
                const int t = __ldcg(u + U_T), sym = __ldcg(u + U_SYM), hb = __ldcg(u + U_HBUF);
                const int nf = __ldcg(u + U_NFRAMES);
                T.s_lst[i] = make_int2(nf - t, sym | (hb << 30));
            }
        }
    }
    __syncthreads();
    tc_prefetch_encp(P, T, nl);
}

// Replicated decision (tensor-core loop, n_live <= kTcRec, no trace): every CTA
// decides every live utterance from the argmax keys and its own shared-memory
// copy of (frames left, symbol count, h buffer), and compacts the next emit and
// live lists in place in shared memory, so no leader round trip, list write-out
// or record reload separates the joint from the next LSTM phase. The decisions
// are the leader's (decide_core on the same keys). The last CTA (the one with
// the fewest rows in every phase) alone applies what the leader writes
// (utterance state, tokens, boundaries, finish times, control words) and clears
// these utterances' entries of the other key buffer, which every CTA finished
// reading one iteration ago and the joint after next fills.
// Returns the next iteration's control word.
__device__ unsigned long long rep_decide(const LoopParams & P, const TcSmem & T, int sel, int n_live,
                                         const unsigned long long * keys, unsigned long long * keys_other) {
    const bool writer = blockIdx.x == gridDim.x - 1;
    const int i = threadIdx.x;   // n_live <= kTcRec == blockDim.x: one entry per thread
    int e = 0, lv = 0, utt = -1, etok = 0, ereset = 0, hb = 0, rem = 0, sym = 0, err = 0;
    long long lframe = 0;
    if (i < n_live) {
        utt = T.s_lutt[i];
        const int2 st = T.s_lst[i];
        int * u = P.ust + utt * kUst;
        // the writer's state loads go out with the key loads (one round trip)
        int4 u0 = make_int4(0, 0, 0, 0), u1 = u0, u2 = u0;
        if (writer) {
            u0 = __ldcg(reinterpret_cast<const int4 *>(u));
            u1 = __ldcg(reinterpret_cast<const int4 *>(u) + 1);
            u2 = __ldcg(reinterpret_cast<const int4 *>(u) + 2);
        }
        const unsigned long long kt = __ldcg(&keys[2 * utt + 0]);
        const unsigned long long kd = P.is_tdt ? __ldcg(&keys[2 * utt + 1]) : 0ull;
        int tok = key_index(kt);
        int di = P.is_tdt ? key_index(kd) : 0;
        if (keys_bad(P, kt, kd, tok, di)) {   // the same keys, so the same verdict, in every CTA
            err = 1;
            if (writer) {
                atomicCAS(&P.ctl[C_ERR], 0, (int) PK_ERR_DEVICE);
                P.ctl[C_ERRINFO] = utt;
            }
            tok = P.blank;
            di = 0;
        }
        const int s0 = st.y & 0x3FFFFFFF;
        hb = (st.y >> 30) & 1;
        const Decision d = decide_core(P, tok, di, s0);
        rem = st.x - d.adv;
        sym = d.sym;
        e = d.e; etok = d.etok; ereset = d.ereset;
        if (e) hb ^= 1;
        lv = rem > 0 ? 1 : 0;
        lframe = T.s_lframe[i] + d.adv;
        if (writer) {
            const int uf[12] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w, u2.x, u2.y, u2.z, u2.w};
            keys_other[2 * utt + 0] = 0ull;
            if (P.is_tdt) keys_other[2 * utt + 1] = 0ull;
            u[U_STEPS] = uf[U_STEPS] + 1;
            int ntok = uf[U_NTOK];
            if (!P.is_tdt) eou_effects(P, u, uf, utt, d, s0, ntok, tok, uf[U_NFRAMES]);
            if (d.emit_tok && !put_token(P, utt, tok, ntok, uf[U_NFRAMES])) err = 1;
            if (e) u[U_HBUF] = hb;
            u[U_T] = uf[U_T] + d.adv;
            u[U_SYM] = sym;
            u[U_NTOK] = ntok;
            if (!lv) P.finish_ns[utt] = gtimer();
        }
    }
    // every thread has read its entry before the scan's first barrier, so the
    // compacted lists can overwrite the current ones in place
    int tot = 0;
    const int pf = block_excl_scan(e | (lv << 16), as_smem(T), tot);
    const int pe = pf & 0xFFFF, pl = pf >> 16;
    const int n_emit = tot & 0xFFFF, n_next = tot >> 16;
    if (e) {
        T.s_utt[pe] = utt;
        T.s_aux[pe] = etok;
        T.s_aux2[pe] = ereset | (hb << 1);
    }
    if (lv) {
        T.s_lutt[pl] = utt;
        T.s_lframe[pl] = lframe;
        T.s_lst[pl] = make_int2(rem, sym | (hb << 30));
    }
    if (writer && threadIdx.x == 0) {
        P.ctl[C_NEMIT] = n_emit;
        P.ctl[C_NLIVE0 + (sel ^ 1)] = n_next;
        P.ctl[C_NDECIDED] = n_live;
        P.ctl[C_SEL] = sel ^ 1;
    }
    const int any_err = __syncthreads_or(err);
    return pack_ctl(0u, any_err, sel ^ 1, n_emit, n_next);
}

template <bool Q8>
__device__ void tc_phase_lstm(const LoopParams & P, int l, int n_emit, const TcSmem & T) {
    const int H = P.H, L = P.L, B = P.B;
    const int upc = P.upc;
    const int u0 = (int) blockIdx.x * upc;
    const int nu = max(0, min(H, u0 + upc) - u0);
    if (nu == 0) return;
    const TcBlock & bk = P.tcl[l];
    const int es = h_es(P);
    const int PR = kTcM * P.mb;                               // utterances per pass
    const unsigned hbytes = (unsigned) (2 * H * es);          // one staged h row: hi | lo
    // state row of (h buffer, layer, utterance) and compact row of (layer, emit index)
    auto hst = [&](int hb, int layer, int utt) -> unsigned char * {
        return P.hst + ((((size_t) hb * L + layer) * B + utt) * P.rbh);
    };
    auto xnew = [&](int layer, int e) -> unsigned char * {
        return P.xnew + (((size_t) layer * B + e) * P.rbh);
    };
    SUBMARK(-1);
    for (int rb = 0; rb < n_emit; rb += kTcRec) {
      const int nrb = min(kTcRec, n_emit - rb);
      if (n_emit > kTcRec) {   // otherwise the records loaded at the start of the iteration are in place
          for (int i = threadIdx.x; i < nrb; i += blockDim.x) tc_emit_record(P, T, i, rb + i);
          __syncthreads();
      }
      SUBMARK(0);
      for (int cs = 0; cs < nrb; cs += PR) {
        const int nc = min(PR, nrb - cs);
        const TcSmem S = tc_pass(T, cs);
        const int mbp = nc > kTcM ? 2 : 1;          // m16 blocks computed for this pass
        // Prefetch the cell-update operands (layer-0 table rows and the old cell
        // state) before the GEMM so their latency overlaps it. One (utterance,
        // unit) pair per thread: nc * nu <= PR * upc <= blockDim. Raw loads only:
        // nothing consumes them before the cell update.
        const int my = threadIdx.x;
        const bool act = my < nc * nu;
        // unit fastest: consecutive threads prefetch consecutive table / state entries
        const int cc = act ? my / nu : 0, jj = act ? my - (my / nu) * nu : 0;
        const int j = u0 + jj;
        float g0v[4] = {0.f, 0.f, 0.f, 0.f};
        float c_old = 0.0f;
        if (act) {
            if (l == 0) {
#pragma unroll
                for (int q = 0; q < 4; ++q) g0v[q] = __ldg(P.g0 + (size_t) S.s_aux[cc] * 4 * H + q * H + j);
            }
            if (!(S.s_aux2[cc] & 1)) c_old = __ldcg(P.c + ((size_t) l * B + S.s_utt[cc]) * H + j);
        }
        SUBMARK(1);
        // h_prev of layer l (zero on reset) goes row by row into the last region;
        // above layer 0 the new h of layer l-1 comes first, one compact tile.
        unsigned char * reg1 = S.area + (size_t) PR * P.rbh;
        const unsigned char * tile = l == 0 ? nullptr : xnew(l - 1, rb + cs);
        if (!tc_stage(P, S, nc, tile, (unsigned) P.rbh, S.area, l == 0 ? S.area : reg1, hbytes, (unsigned) P.rbh,
                      [&](int c) -> const unsigned char * {
                          const int utt = S.s_utt[c], a2 = S.s_aux2[c];
                          if (a2 & 1) return nullptr;
                          return hst((a2 >> 1) ^ 1, l, utt);
                      })) return;
        ATile A;
        A.r0 = S.area;
        A.r1 = reg1;
        A.rb = P.rbh;
        A.lo = H * es;
        A.kb_split = l == 0 ? (bk.K >> 5) : (H >> 5);
        if constexpr (Q8) {
            q8_rows(S.area, nc, P.rbh, H, A.lo, true, false);
            if (l > 0) q8_rows(reg1, nc, P.rbh, H, A.lo, true, false);
        }
        tc_gemm_q<Q8>(P, S, bk, 0, bk.tiles, A, mbp, 4,
                l == 0 ? nc * P.rbh : PR * P.rbh + nc * P.rbh);
        SUBMARK(3);
        // cell update (parakeet_tdt.cpp:123-136); block row = unit * 4 + gate
        if (act) {
            const int utt = S.s_utt[cc];
            const int hb = S.s_aux2[cc] >> 1;
            float gate[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int row = jj * 4 + q;
                // ((b_ih + W_ih x) + b_hh) + W_hh h, with b_ih + W_ih x for layer 0 from
                // the table; S.lb holds b_hh for layer 0 and b_ih + b_hh above it
                const float pre = (l == 0 ? g0v[q] : 0.0f) + S.lb[(l * 4 + q) * upc + jj];
                gate[q] = pre + S.C[c_index(row, cc, kTcM * mbp)];
            }
            const float i_g = sigmoid_ref(gate[0]);
            const float f_g = sigmoid_ref(gate[1]);
            const float g_g = tanhf(gate[2]);
            const float o_g = sigmoid_ref(gate[3]);
            const float c_new = f_g * c_old + i_g * g_g;
            P.c[((size_t) l * B + utt) * H + j] = c_new;
            const float hn = o_g * tanhf(c_new);
            P.h[(((size_t) hb * L + l) * B + utt) * H + j] = hn;
            put_h(P, hst(hb, l, utt), j, hn);
            put_h(P, xnew(l, rb + cs + cc), j, hn);
        }
        __syncthreads();
        SUBMARK(4);
      }
    }
}

template <bool Q8>
__device__ void tc_phase_pred(const LoopParams & P, bool first, int n_emit, int sel, int n_live,
                              const TcSmem & T) {
    const int H = P.H, J = P.J, L = P.L, B = P.B;
    const int rpc = P.rpc_p;
    const int j0 = (int) blockIdx.x * rpc;
    const int nr = max(0, min(J, j0 + rpc) - j0);
    const int * live = P.live + (size_t) sel * B;
    const int n_list = first ? n_live : n_emit;
    const int es = h_es(P);
    const int PR = kTcM * P.mb;                 // utterances per pass
    SUBMARK(-1);
    if (nr > 0) {
      for (int rb = 0; rb < n_list; rb += kTcRec) {
        const int nrb = min(kTcRec, n_list - rb);
        // records hold the h buffer as s_aux2 >> 1 (the LSTM's record format); after
        // the first iteration, a list that fits one block is already in place
        if (first || n_list > kTcRec) {
            for (int i = threadIdx.x; i < nrb; i += blockDim.x) {
                if (first) {
                    const int utt = __ldcg(&live[rb + i]);
                    T.s_utt[i] = utt;
                    T.s_aux2[i] = __ldcg(&P.ust[utt * kUst + U_HBUF]) << 1;
                } else {
                    tc_emit_record(P, T, i, rb + i);
                }
            }
            __syncthreads();
        }
        SUBMARK(5);
        for (int cs = 0; cs < nrb; cs += PR) {
            const int nc = min(PR, nrb - cs);
            const TcSmem S = tc_pass(T, cs);
            const int mbp = nc > kTcM ? 2 : 1;          // m16 blocks computed for this pass
            const int TG = mbp == 2 ? 7 : kTcRmax;      // weight tiles per GEMM call
            // after the first iteration the pred list is the emit list: the last
            // layer's new h is one compact tile; on the first iteration (the live
            // list) rows come from the state, one by one
            bool staged;
            if (first) {
                staged = tc_stage(P, S, nc, nullptr, 0u, S.area, S.area, (unsigned) (2 * H * es), (unsigned) P.rbh,
                                  [&](int c) -> const unsigned char * {
                                      return P.hst + ((((size_t) (S.s_aux2[c] >> 1) * L + (L - 1)) * B + S.s_utt[c]) * P.rbh);
                                  });
            } else {
                staged = tc_stage(P, S, nc, P.xnew + (((size_t) (L - 1) * B + rb + cs) * P.rbh), (unsigned) P.rbh,
                                  S.area, nullptr, 0u, 0u, [&](int) -> const unsigned char * { return nullptr; });
            }
            if (!staged) return;
            ATile A;
            A.r0 = A.r1 = S.area;
            A.rb = P.rbh;
            A.lo = H * es;
            A.kb_split = P.tcp.K >> 5;
            if constexpr (Q8) q8_rows(S.area, nc, P.rbh, H, A.lo, true, false);
            for (int t0 = 0; t0 < P.tcp.tiles; t0 += TG) {
                const int nt = min(TG, P.tcp.tiles - t0);
                tc_gemm_q<Q8>(P, S, P.tcp, t0, nt, A, mbp, mbp == 2 ? kWarps : 4, nc * P.rbh);
                for (int idx = threadIdx.x; idx < nc * nt * 8; idx += blockDim.x) {
                    const int rr = idx / nc, cc = idx - rr * nc, row = t0 * 8 + rr;   // utterance fastest
                    if (row < nr) {
                        const int r = row - t0 * 8;
                        const int j = j0 + row;
                        P.predp[(size_t) S.s_utt[cc] * J + j] = S.bp[row] + S.C[c_index(r, cc, kTcM * mbp)];
                    }
                }
                __syncthreads();
                SUBMARK(7);
            }
        }
      }
        if (n_live <= kTcRec) joint_hidden(P, sel, n_live, j0, nr, T.s_lutt, T.s_lframe);
        else joint_hidden(P, sel, n_live, j0, nr);
        SUBMARK(8);
    }
    trace_state_dump(P, first, sel);
}

// Joint epilogue of one GEMM call: logits = bias + C for this CTA's rows, the
// best (token, duration) key per utterance max-reduced into keys. Thread =
// (utterance c, row group rg): consecutive threads read consecutive C columns;
// row-group partial keys meet in the staging area (free again once C is
// reduced), then one thread per utterance folds them (unrolled, loads in
// flight together) into the global keys. W = utterance columns of C.
template <int W>
__device__ __forceinline__ void joint_keys(const LoopParams & P, const TcSmem & S, int nc, int nt, int t0, int nr,
                                           int r0, unsigned long long * keys) {
    constexpr int RG = kThreads / W;
    const int c = threadIdx.x % W, rg = threadIdx.x / W;
    unsigned long long bt = 0ull, bd = 0ull;
    if (c < nc) {
        for (int rr = rg; rr < nt * 8; rr += RG) {
            const int row = t0 * 8 + rr;
            if (row >= nr) break;
            const int r = r0 + row;
            const float logit = S.bj[row] + S.C[c_index(rr, c, W)];
            if (P.trace_steps > 0) {
                const int step = S.s_aux[c];
                if (step < P.trace_steps)
                    P.tr_logits[((size_t) S.s_utt[c] * P.trace_steps + step) * P.Vo + r] = logit;
            }
            if (r < P.V1) {
                const unsigned long long k = make_key(logit, r);
                bt = k > bt ? k : bt;
            } else {
                const unsigned long long k = make_key(logit, r - P.V1);
                bd = k > bd ? k : bd;
            }
        }
    }
    // (at the end of the area: with several calls per pass, the staged rows at its
    // start feed the next one)
    ulonglong2 * kp = reinterpret_cast<ulonglong2 *>(S.area + ((P.area - kThreads * 16) & ~15));
    kp[threadIdx.x] = make_ulonglong2(bt, bd);
    SUBMARK(18);
    __syncthreads();
    SUBMARK(19);
    if (threadIdx.x < nc) {
#pragma unroll
        for (int g = 1; g < RG; ++g) {
            const ulonglong2 o = kp[g * W + threadIdx.x];
            bt = o.x > bt ? o.x : bt;
            bd = o.y > bd ? o.y : bd;
        }
    }
    // generic accesses of the area before the next stage's bulk writes; ahead of
    // the global reductions so that it does not wait for them
    SUBMARK(20);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    SUBMARK(21);
    if (threadIdx.x < nc) {
        const int utt = S.s_utt[threadIdx.x];
        if (bt) atomicMax(&keys[2 * utt + 0], bt);
        if (bd) atomicMax(&keys[2 * utt + 1], bd);
    }
    SUBMARK(22);
}

template <bool Q8>
__device__ void tc_phase_joint(const LoopParams & P, int sel, int n_live, const TcSmem & T, unsigned long long * keys) {
    const int J = P.J, B = P.B;
    const int rpc = P.rpc_j;
    const int r0 = (int) blockIdx.x * rpc;
    const int nr = max(0, min(P.Vo, r0 + rpc) - r0);
    if (nr == 0) return;
    const int * live = P.live + (size_t) sel * B;
    const int PR = kTcM * P.mb;                 // utterances per pass
    SUBMARK(-1);
    for (int rb = 0; rb < n_live; rb += kTcRec) {
      const int nrb = min(kTcRec, n_live - rb);
      // a live list that fits one block was loaded at the start of the iteration
      if (n_live > kTcRec || P.trace_steps > 0) {
          for (int i = threadIdx.x; i < nrb; i += blockDim.x) {
              const int utt = n_live > kTcRec ? __ldcg(&live[rb + i]) : T.s_lutt[i];
              T.s_utt[i] = utt;
              if (P.trace_steps > 0) T.s_aux[i] = __ldcg(&P.ust[utt * kUst + U_STEPS]);
          }
          __syncthreads();
      }
      int * lrec = (n_live > kTcRec || P.trace_steps > 0) ? T.s_utt : T.s_lutt;
      SUBMARK(9);
      for (int cs = 0; cs < nrb; cs += PR) {
        const int nc = min(PR, nrb - cs);
        TcSmem S = tc_pass(T, cs);
        S.s_utt = lrec + cs;
        const int mbp = nc > kTcM ? 2 : 1;              // m16 blocks computed for this pass
        const int TG = mbp == 2 ? 7 : kTcRmax;          // weight tiles per GEMM call
        // the joint hidden rows of this pass: one compact tile (live-list order)
        if (!tc_stage(P, S, nc, P.hidc + (size_t) (rb + cs) * P.rbj, (unsigned) P.rbj, S.area, nullptr, 0u, 0u,
                      [&](int) -> const unsigned char * { return nullptr; })) return;
        ATile A;
        A.r0 = A.r1 = S.area;
        A.rb = P.rbj;
        A.lo = J * 2;
        A.kb_split = P.tcj.K >> 5;
        if constexpr (Q8) q8_rows(S.area, nc, P.rbj, J, A.lo, false, true);
        for (int t0 = 0; t0 < P.tcj.tiles; t0 += TG) {
            const int nt = min(TG, P.tcj.tiles - t0);
            tc_gemm_q<Q8>(P, S, P.tcj, t0, nt, A, mbp, 4, nc * P.rbj);
            SUBMARK(11);
            if (mbp == 2) joint_keys<2 * kTcM>(P, S, nc, nt, t0, nr, r0, keys);
            else joint_keys<kTcM>(P, S, nc, nt, t0, nr, r0, keys);
            __syncthreads();
            SUBMARK(12);
        }
      }
    }
}

// Copy this CTA's slice of every tensor-core weight block into shared memory.
__device__ void tc_load_stationary(const LoopParams & P, const TcSmem & T) {
    auto copy = [&](unsigned dst_off, const void * src, unsigned bytes) {
        const uint4 * s4 = reinterpret_cast<const uint4 *>(src);
        uint4 * d4 = reinterpret_cast<uint4 *>(T.w + dst_off);
        for (unsigned i = threadIdx.x; i < bytes / 16; i += blockDim.x) d4[i] = __ldg(s4 + i);
    };
    auto block = [&](const TcBlock & b) {
        copy(b.sm_frag, b.frag + (size_t) blockIdx.x * b.cta_bytes, b.cta_bytes);
        if (b.is_i8) copy(b.sm_scale, b.scale + (size_t) blockIdx.x * b.cta_scales, b.cta_scales * 4u);
    };
    block(P.tcj);
    block(P.tcp);
    for (int l = 0; l < P.L; ++l) block(P.tcl[l]);
    __syncthreads();
}

// Q8: PK_MATH_Q8 (its own instantiation, so that the default kernel's register
// allocation does not carry the q8_0-activation code).
template <bool TC, bool Q8>
__global__ void __launch_bounds__(kThreads, 1) step_loop_kernel(const LoopParams P) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem S;
    TcSmem T;
    if constexpr (TC) {
        T = tc_carve(smem_raw, P);
        S = as_smem(T);
    } else {
        const int upc = (P.H + (int) gridDim.x - 1) / (int) gridDim.x;
        S = carve(smem_raw, P, upc);
    }
    unsigned gen = 0u;   // leader generations; the host zeroes the barrier words before every launch
    unsigned nbar = 0u;  // counter barriers passed
    if (blockIdx.x == 0 && threadIdx.x == 0 && !P.resume) *P.t_start = gtimer();
    // a batch continued from the bulk loop counts its iterations on from there
    // (only CTA 0's thread 0 reads and writes these words)
    int iter_base = 0, emit_base = 0;
    if (P.resume && blockIdx.x == 0 && threadIdx.x == 0) {
        iter_base = __ldcg(&P.ctl[C_ITERS]);
        emit_base = __ldcg(&P.ctl[C_EMITITERS]);
    }
    // Test hook (PK_OPT_TEST_STALL): CTA 0 never arrives, every other CTA's
    // first barrier wait runs out after timeout_ns and records PK_ERR_TIMEOUT.
    if (P.test_stall && blockIdx.x == 0) return;
    if constexpr (TC) {
        // activation rows that a pass does not stage keep finite (zero) values
        for (int i = threadIdx.x; i < P.area / 16; i += blockDim.x)
            reinterpret_cast<uint4 *>(T.area)[i] = make_uint4(0u, 0u, 0u, 0u);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (threadIdx.x == 0) {
            const unsigned mb = (unsigned) __cvta_generic_to_shared(T.mbar);
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(mb), "r"(kWarps) : "memory");
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            T.s_flag[2] = 0;   // staging barrier phase
        }
        for (int i = threadIdx.x; i < P.rpc_j; i += blockDim.x) {
            const int r = (int) blockIdx.x * P.rpc_j + i;
            T.bj[i] = r < P.Vo ? __ldg(P.out_b + r) : 0.0f;
        }
        for (int i = threadIdx.x; i < P.rpc_p; i += blockDim.x) {
            const int j = (int) blockIdx.x * P.rpc_p + i;
            T.bp[i] = j < P.J ? __ldg(P.pred_b + j) : 0.0f;
        }
        for (int i = threadIdx.x; i < P.L * 4 * P.upc; i += blockDim.x) {
            const int l = i / (4 * P.upc), q = (i / P.upc) % 4, jj = i % P.upc;
            const int j = (int) blockIdx.x * P.upc + jj;
            float v = 0.0f;
            if (j < P.H) {
                const int gr = q * P.H + j;
                v = l == 0 ? __ldg(P.b_hh[0] + gr) : __ldg(P.b_ih[l] + gr) + __ldg(P.b_hh[l] + gr);
            }
            T.lb[i] = v;
        }
        __syncthreads();
        if (P.stationary) tc_load_stationary(P, T);
    }
    SUBMARK(-3);
    bool first = true;
    bool rep = false;    // lists and control state held in shared memory (replicated decisions)
    int emit_iters = 0;
    // CTA 0 timestamps: per segment, its own work and the wait that follows
    // (accumulators in shared memory: registers are the loop's scarcest resource)
    __shared__ unsigned long long pacc[9];   // 8 segments, then the last timestamp
    const bool prof = blockIdx.x == 0 && threadIdx.x == 0 && P.prof != nullptr;
    if (prof) {
        for (int i = 0; i < 8; ++i) pacc[i] = 0ull;
        pacc[8] = gtimer();
    }
    auto mark = [&](int slot) {
        if (prof) {
            const unsigned long long now = gtimer();
            pacc[slot] += now - pacc[8];
            pacc[8] = now;
        }
    };
    // control state of the first iteration from the host-written words; later
    // ones arrive with the leader's release word
    unsigned long long cw;
    {
        const int4 cw0 = __ldcg(reinterpret_cast<const int4 *>(P.ctl));
        const int4 cw1 = __ldcg(reinterpret_cast<const int4 *>(P.ctl) + 1);
        cw = pack_ctl(0u, cw0.x, cw0.y, cw1.x, cw0.y ? cw0.w : cw0.z);
    }
    for (int iter = 0;; ++iter) {
        // Every utterance advances its frame pointer at least once per
        // (max_sym + 1) iterations, so this bound only trips on a bug.
        if (iter > P.max_iters) {
            if (blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(&P.ctl[C_ERR], 0, (int) PK_ERR_DEVICE);
            return;
        }
        if ((cw >> 47) & 1ull) return;          // error flagged
        const int sel = (int) ((cw >> 46) & 1ull);
        const int n_emit = (int) ((cw >> 23) & 0x7FFFFFull);
        const int n_live = (int) (cw & 0x7FFFFFull);
        if (blockIdx.x == 0 && threadIdx.x == 0 && iter > 0) {
            // plain stores (no read back): decided rounds so far, and how many of them emitted
            P.ctl[C_ITERS] = iter_base + iter;
            if (n_emit > 0) P.ctl[C_EMITITERS] = emit_base + (++emit_iters);
        }
        // this iteration's argmax key buffer (two, alternating)
        unsigned long long * keys = P.keys + (size_t) (iter & 1) * 2 * P.B;
        if constexpr (TC) {
            if (!rep) tc_load_records(P, T, sel, n_emit, n_live);
        }
        if (n_emit > 0) {
            for (int l = 0; l < P.L; ++l) {
                if constexpr (TC) tc_phase_lstm<Q8>(P, l, n_emit, T);
                else phase_lstm(P, l, n_emit, S);
                mark(0);
                if (!grid_barrier(P, nbar, S)) return;
                mark(1);
            }
        }
        if constexpr (TC) tc_phase_pred<Q8>(P, first, n_emit, sel, n_live, T);
        else phase_pred(P, first, n_emit, sel, n_live, S);
        mark(2);
        if (!grid_barrier(P, nbar, S)) return;
        mark(3);
        first = false;
        if (n_live == 0) break;
        if constexpr (TC) tc_phase_joint<Q8>(P, sel, n_live, T, keys);
        else phase_joint(P, sel, n_live, S, keys);
        mark(4);
        bool rep_now = false;
        if constexpr (TC) rep_now = rep_mode(P, n_live);
        if (rep_now) {
            if (!grid_barrier(P, nbar, S)) return;
            mark(5);
            SUBMARK(-4);
            cw = rep_decide(P, T, sel, n_live, keys, P.keys + (size_t) ((iter + 1) & 1) * 2 * P.B);
            SUBMARK(13);
            tc_prefetch_encp(P, T, (int) (cw & 0x7FFFFFull));
            rep = true;
            mark(6);
        } else if (leader_arrive(P, S)) {
            SUBMARK(-4);
            const int * lsm = nullptr;
            if constexpr (TC) lsm = n_live <= kTcRec ? T.s_lutt : nullptr;
            cw = leader_decide(P, S, sel, n_live, gen + 1u, keys, lsm);
            SUBMARK(13);
            mark(6);
            leader_release(P, cw);
        } else if (!leader_wait(P, gen, S, cw)) {
            return;
        }
        mark(7);
        ++gen;
    }
    SUBMARK(-2);
    if (prof)
        for (int i = 0; i < 8; ++i) P.prof[i] = pacc[i];
}

}  // namespace

size_t step_loop_smem_bytes(int chunk, int ldx, int H, int grid) {
    const int upc = (H + grid - 1) / grid;
    size_t off = (size_t) chunk * ldx * sizeof(float);
    off += (size_t) chunk * upc * 4 * sizeof(float);
    off = (off + 15) & ~(size_t) 15;
    off += (size_t) kWarps * 32 * 2 * sizeof(unsigned long long);
    off += 3 * 32 * sizeof(int) + (kWarps + 2) * sizeof(int) + 8 * sizeof(int);
    return off;
}

size_t step_loop_tc_smem_bytes(unsigned sm_weights, int area, int rpc_j, int rpc_p, int upc) {
    size_t off = (sm_weights + 15) & ~15u;
    off += (size_t) area;
    off += (size_t) kTcRmax * 128 * 2 * 4;
    off += 16;
    off += 4 * kTcRec * 4 + 2 * kTcRec * 8 + (kWarps + 2) * 4 + 8 * 4;
    off += (size_t) (rpc_j + rpc_p) * 4;
    off += (size_t) kMaxLayers * 4 * upc * 4;
    return off;
}

cudaError_t step_loop_configure(size_t smem, int tc) {
    if (!tc) return cudaFuncSetAttribute(step_loop_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    const cudaError_t e = cudaFuncSetAttribute(step_loop_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int) smem);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(step_loop_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
}

size_t step_loop_static_smem(int tc) {
    cudaFuncAttributes a{};
    cudaFuncAttributes q{};
    const cudaError_t e = tc ? cudaFuncGetAttributes(&a, step_loop_kernel<true, false>)
                             : cudaFuncGetAttributes(&a, step_loop_kernel<false, false>);
    if (e != cudaSuccess) return 0;
    if (tc && cudaFuncGetAttributes(&q, step_loop_kernel<true, true>) == cudaSuccess)
        return a.sharedSizeBytes > q.sharedSizeBytes ? a.sharedSizeBytes : q.sharedSizeBytes;
    return a.sharedSizeBytes;
}

cudaError_t step_loop_occupancy(size_t smem, int tc, int * blocks_per_sm) {
    if (!tc) return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, step_loop_kernel<false, false>, kThreads, smem);
    int a = 0, q = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&a, step_loop_kernel<true, false>, kThreads, smem);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&q, step_loop_kernel<true, true>, kThreads, smem);
    *blocks_per_sm = a < q ? a : q;
    return e;
}

cudaError_t launch_step_loop(const LoopParams & p, int grid, size_t smem, cudaStream_t s) {
    void * args[] = {const_cast<LoopParams *>(&p)};
    const void * fn = !p.tc ? reinterpret_cast<const void *>(step_loop_kernel<false, false>)
                      : p.q8 ? reinterpret_cast<const void *>(step_loop_kernel<true, true>)
                             : reinterpret_cast<const void *>(step_loop_kernel<true, false>);
    return cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kThreads), args, smem, s);
}

}  // namespace pk

#ifdef PK_SUBPROF
// Development builds only: the sub-phase cycle counters of the last launch.
extern "C" __attribute__((visibility("default"))) int pk_debug_subprof(unsigned long long * out) {
    return (int) cudaMemcpyFromSymbol(out, pk::g_subprof, sizeof(unsigned long long) * 24);
}
#endif
