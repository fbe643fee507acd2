// pk_device.cuh -- device helpers shared by the step-loop kernels of
// libparakeet_cuda (pk_loop.cu: the persistent loop; pk_bulk.cu: the
// tensor-memory loop for large live batches): timers and ordered global
// accesses, the argmax key, the greedy control of one utterance's step and the
// staged layout of h rows.
#pragma once

#include "pk_internal.h"

#include <cuda_fp16.h>
#include <math.h>

namespace pk {
namespace {

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned * p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned long long * p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release64(unsigned long long * p, unsigned long long v) {
    asm volatile("st.release.gpu.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}

// Arrival without waiting for the old value (fire-and-forget, release ordered).
__device__ __forceinline__ void red_add_release(unsigned * p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned * p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Order-preserving 64-bit argmax key: larger value wins, then the smaller index
// (the reference's strict '>' keeps the first maximum). -0 is folded onto +0
// because the reference compares them equal.
__device__ __forceinline__ unsigned long long make_key(float v, int idx) {
    unsigned u = __float_as_uint(v);
    if (u == 0x80000000u) u = 0u;
    const unsigned ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long) ord << 32) | (unsigned long long) (0xFFFFFFFFu - (unsigned) idx);
}
__device__ __forceinline__ int key_index(unsigned long long k) {
    return (int) (0xFFFFFFFFu - (unsigned) (k & 0xFFFFFFFFull));
}

__device__ __forceinline__ float sigmoid_ref(float x) { return 1.0f / (1.0f + expf(-x)); }

// The leader's release word (P.bar[4..5]) carries the next iteration's control
// state, so the waiters need no further load: generation (16 bits) << 48 |
// error << 47 | list selector << 46 | emit count << 23 | live count.
__device__ __forceinline__ unsigned long long pack_ctl(unsigned gen, int err, int sel, int n_emit, int n_live) {
    return ((unsigned long long) (gen & 0xFFFFu) << 48) | ((unsigned long long) (err != 0) << 47) |
           ((unsigned long long) (sel & 1) << 46) | ((unsigned long long) (unsigned) n_emit << 23) |
           (unsigned long long) (unsigned) n_live;
}

// ---- greedy control ---------------------------------------------------------

// One utterance's step for the decided (token, duration index) and its current
// symbol count: frame advance, new symbol count and the emit record.
//  * TDT, parakeet_tdt.cpp:938-968: blank advances by max(1, dur); a token is
//    emitted and advances when dur > 0 or max_symbols is reached.
//  * EOU, parakeet_eou.cpp:271-333: blank / EOB / a special piece end the frame;
//    EOU ends the frame, resets the prediction net (re-primed on blank) and may
//    record a boundary; any other token is emitted. kind tells the state writer
//    which side effects follow: 0 frame end, 1 end of utterance, 2 token,
//    3 token that reaches max_symbols (and ends the frame).
struct Decision {
    int adv, sym, e, etok, ereset, emit_tok, kind;
};

__device__ __forceinline__ Decision decide_core(const LoopParams & P, int tok, int di, int s0) {
    Decision d{0, s0, 0, 0, 0, 0, 0};
    const int msym = P.max_sym;
    if (P.is_tdt) {
        const int dur = P.Nd > 0 ? __ldg(P.durations + di) : di;
        const int adv = dur > 1 ? dur : 1;
        if (tok == P.blank) {
            d.adv = adv; d.sym = 0;
        } else {
            d.emit_tok = 1; d.e = 1; d.etok = tok;
            ++d.sym;
            if (dur > 0 || d.sym >= msym) { d.adv = adv; d.sym = 0; }
        }
    } else if (tok == P.blank || tok == P.eob) {
        d.adv = 1; d.sym = 0;
    } else if (tok == P.eou) {
        d.kind = 1; d.e = 1; d.etok = P.blank; d.ereset = 1; d.adv = 1; d.sym = 0;
    } else if (tok < P.n_special && __ldg(P.special + tok)) {
        d.adv = 1; d.sym = 0;
    } else {
        d.kind = 2; d.emit_tok = 1; d.e = 1; d.etok = tok;
        ++d.sym;
        if (d.sym >= msym) { d.kind = 3; d.adv = 1; d.sym = 0; }
    }
    return d;
}

// EOU state side effects of a decision (uf: the utterance's state before it).
// The frame loop resets symbols_this_step at each frame start; U_SYMX keeps the
// value a frame ended with (what the reference's state holds after the window).
__device__ __forceinline__ void eou_effects(const LoopParams & P, int * u, const int * uf, int utt,
                                            const Decision & d, int s0, int ntok, int tok, int T) {
    if (d.kind == 0) {
        u[U_SYMX] = s0;
    } else if (d.kind == 1) {
        u[U_SYMX] = s0;
        const int total = uf[U_NBEFORE] + ntok;
        if (total > uf[U_SEGSTART]) {
            const int nb = uf[U_NBND];
            if (P.bnd_out != nullptr && nb < T) P.bnd_out[P.bnd_region[utt] + nb] = total;
            u[U_NBND] = nb + 1;
            u[U_SEGSTART] = total;
        }
        u[U_LAST] = P.blank;
    } else {
        u[U_LAST] = tok;
        if (d.kind == 3) u[U_SYMX] = s0 + 1;
    }
}

// An argmax key that no joint row produced, or an index out of range.
__device__ __forceinline__ bool keys_bad(const LoopParams & P, unsigned long long kt, unsigned long long kd,
                                         int tok, int di) {
    return kt == 0ull || tok < 0 || tok >= P.V1 || (P.is_tdt && (kd == 0ull || di < 0 || di >= P.Nd));
}

// Append an emitted token to the utterance's output region; false (error
// flagged) when the region (T * max_symbols tokens) is full.
__device__ __forceinline__ bool put_token(const LoopParams & P, int utt, int tok, int & ntok, int T) {
    const int cap = T * (P.max_sym > 0 ? P.max_sym : 1);
    if (ntok < cap) {
        P.tok_out[P.tok_region[utt] + ntok] = tok;
        ++ntok;
        return true;
    }
    atomicCAS(&P.ctl[C_ERR], 0, (int) PK_ERR_DEVICE);
    P.ctl[C_ERRINFO] = utt;
    return false;
}

// Bytes per h element and the h row layout: [hi | lo] parts of H elements each.
__device__ __forceinline__ int h_es(const LoopParams & P) { return P.h_int ? 1 : 2; }

// Write one new h value into a staged-layout row (state row or compact row).
__device__ __forceinline__ void put_h(const LoopParams & P, unsigned char * row, int j, float hn) {
    if (P.h_int) {
        // int16 fixed point (|h| < 1): signed high digit, unsigned low digit
        const int q16 = max(-32767, min(32767, __float2int_rn(hn * 32768.0f)));
        row[j] = (unsigned char) (int8_t) (q16 >> 8);
        row[P.H + j] = (unsigned char) (q16 & 255);
    } else {
        const __half hh = __float2half_rn(hn);
        reinterpret_cast<__half *>(row)[j] = hh;
        reinterpret_cast<__half *>(row)[P.H + j] = __float2half_rn(hn - __half2float(hh));
    }
}

// Bring bytes (a multiple of 16, 16-byte aligned) at p into L2, no completion tracked.
__device__ __forceinline__ void prefetch_l2(const void * p, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(p), "r"(bytes) : "memory");
}


}  // namespace
}  // namespace pk
