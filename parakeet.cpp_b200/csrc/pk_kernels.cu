// pk_kernels.cu -- load-time dequantisation, the f32 SIMT enc-proj GEMM and the
// token compaction kernels of libparakeet_cuda.

#include "pk_internal.h"

#include <algorithm>

#include <cuda_fp16.h>

namespace pk {
namespace {

// GGUF block formats (public): F16 = binary16; Q8_0 = 32-weight blocks of
// {binary16 d; int8 qs[32]} with value f32(d) * qs[i]. Both are exact in f32,
// as ggml's to_float is (used by the reference at parakeet_tdt.cpp:78-95).
__global__ void dequant_kernel(const uint8_t * __restrict__ src, int type, int64_t n,
                               float * __restrict__ dst) {
    const int64_t stride = (int64_t) gridDim.x * blockDim.x;
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float v;
        if (type == PK_GGML_F32) {
            v = reinterpret_cast<const float *>(src)[i];
        } else if (type == PK_GGML_F16) {
            v = __half2float(reinterpret_cast<const __half *>(src)[i]);
        } else {
            const int64_t blk = i >> 5;
            const int j = (int) (i & 31);
            const uint8_t * b = src + blk * 34;
            const unsigned short dbits = (unsigned short) (b[0] | (b[1] << 8));
            const float d = __half2float(__ushort_as_half(dbits));
            v = (float) (int8_t) b[2 + j] * d;
        }
        dst[i] = v;
    }
}

// out[f][j] = b[j] + sum_k enc[f][k] * w[j][k]   (joint.enc over a whole batch
// of frames; the reference's GPU path runs the same projection once per window,
// build_enc_proj_graph, parakeet_tdt.cpp:433-483). 64x64 tiles, 4x4 per thread.
constexpr int GB_M = 64, GB_N = 64, GB_K = 16;

// VEC: A and W rows start on 16-byte boundaries (base aligned, K % 4 == 0), so
// 4-float loads are used; otherwise every load is a scalar one (a caller's
// device buffer need only be float-aligned).
template <bool VEC>
__global__ void __launch_bounds__(256) encproj_f32_kernel(const float * __restrict__ A, int64_t M,
                                                          int K, const float * __restrict__ W,
                                                          const float * __restrict__ bias, int N,
                                                          float * __restrict__ out) {
    __shared__ __align__(16) float As[GB_K][GB_M + 4];
    __shared__ __align__(16) float Bs[GB_K][GB_N + 4];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = (int64_t) blockIdx.x * GB_M;
    const int n0 = blockIdx.y * GB_N;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    const int lr = tid >> 2;          // 0..63 row of the tile to load
    const int lk = (tid & 3) * 4;     // 0,4,8,12
    for (int k0 = 0; k0 < K; k0 += GB_K) {
        {
            const int64_t m = m0 + lr;
            const int k = k0 + lk;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m < M) {
                const float * p = A + m * K;
                if (VEC && k + 3 < K) {
                    v = __ldg(reinterpret_cast<const float4 *>(p + k));
                } else {
                    if (k < K) v.x = p[k];
                    if (k + 1 < K) v.y = p[k + 1];
                    if (k + 2 < K) v.z = p[k + 2];
                    if (k + 3 < K) v.w = p[k + 3];
                }
            }
            As[lk + 0][lr] = v.x; As[lk + 1][lr] = v.y; As[lk + 2][lr] = v.z; As[lk + 3][lr] = v.w;
        }
        {
            const int n = n0 + lr;
            const int k = k0 + lk;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (n < N) {
                const float * p = W + (int64_t) n * K;
                if (VEC && k + 3 < K) {
                    v = __ldg(reinterpret_cast<const float4 *>(p + k));
                } else {
                    if (k < K) v.x = p[k];
                    if (k + 1 < K) v.y = p[k + 1];
                    if (k + 2 < K) v.z = p[k + 2];
                    if (k + 3 < K) v.w = p[k + 3];
                }
            }
            Bs[lk + 0][lr] = v.x; Bs[lk + 1][lr] = v.y; Bs[lk + 2][lr] = v.z; Bs[lk + 3][lr] = v.w;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < GB_K; ++kk) {
            const float4 a = *reinterpret_cast<const float4 *>(&As[kk][ty * 4]);
            const float4 b = *reinterpret_cast<const float4 *>(&Bs[kk][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w};
            const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n < N) out[m * N + n] = __ldg(bias + n) + acc[i][j];
        }
    }
}

// offsets[0] = 0, offsets[b+1] = offsets[b] + ust[b][field]  (one block).
__global__ void scan_counts_kernel(const int32_t * __restrict__ ust, int B, int field,
                                   int64_t * __restrict__ offsets) {
    __shared__ int64_t warp_sums[32];
    __shared__ int64_t carry;
    if (threadIdx.x == 0) { carry = 0; offsets[0] = 0; }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int base = 0; base < B; base += blockDim.x) {
        const int b = base + threadIdx.x;
        const int64_t v = b < B ? (int64_t) ust[(size_t) b * kUst + field] : 0;
        int64_t x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_sums[warp] = x;
        __syncthreads();
        if (warp == 0) {
            const int nw = blockDim.x / 32;
            const int64_t w = lane < nw ? warp_sums[lane] : 0;
            int64_t y = w;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t z = __shfl_up_sync(0xFFFFFFFFu, y, o);
                if (lane >= o) y += z;
            }
            if (lane < nw) warp_sums[lane] = y - w;
        }
        __syncthreads();
        const int64_t incl = carry + warp_sums[warp] + x;
        if (b < B) offsets[b + 1] = incl;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry = incl;
        __syncthreads();
    }
}

__global__ void gather_kernel(const int32_t * __restrict__ ust, int field,
                              const int32_t * __restrict__ src, const int64_t * __restrict__ region,
                              const int64_t * __restrict__ offsets, int32_t * __restrict__ dst) {
    const int b = blockIdx.x;
    const int n = ust[(size_t) b * kUst + field];
    const int32_t * s = src + region[b];
    int32_t * d = dst + offsets[b];
    for (int i = threadIdx.x; i < n; i += blockDim.x) d[i] = s[i];
}

__global__ void split_f16_kernel(const float * __restrict__ src, __half * __restrict__ hi,
                                 __half * __restrict__ lo, int64_t n) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float x = src[i];
    const __half h = __float2half_rn(x);
    hi[i] = h;
    lo[i] = __float2half_rn(x - __half2float(h));
}

__global__ void split_int16_kernel(const float * __restrict__ src, int8_t * __restrict__ hi,
                                   uint8_t * __restrict__ lo, int64_t n) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int q = max(-32767, min(32767, __float2int_rn(src[i] * 32768.0f)));
    hi[i] = (int8_t) (q >> 8);
    lo[i] = (uint8_t) (q & 255);
}

__global__ void stage_rows_kernel(const float * __restrict__ src, int n_rows, int H, int es, int rb,
                                  unsigned char * __restrict__ dst) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows * H) return;
    const int r = i / H, j = i - (i / H) * H;
    const float x = src[i];
    unsigned char * row = dst + (size_t) r * rb;
    if (es == 1) {
        const int q = max(-32767, min(32767, __float2int_rn(x * 32768.0f)));
        row[j] = (unsigned char) (int8_t) (q >> 8);
        row[H + j] = (unsigned char) (q & 255);
    } else {
        const __half h = __float2half_rn(x);
        reinterpret_cast<__half *>(row)[j] = h;
        reinterpret_cast<__half *>(row)[H + j] = __float2half_rn(x - __half2float(h));
    }
}

__global__ void extract_field_kernel(const int32_t * __restrict__ ust, int B, int field,
                                     int32_t * __restrict__ dst) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) dst[b] = ust[(size_t) b * kUst + field];
}

}  // namespace

cudaError_t launch_dequant(const void * src, int type, int64_t ne0, int64_t rows, float * dst,
                           cudaStream_t s) {
    const int64_t n = ne0 * rows;
    if (n <= 0) return cudaSuccess;
    const int threads = 256;
    const int64_t want = (n + threads - 1) / threads;
    const int blocks = (int) (want < 65536 ? want : 65536);
    dequant_kernel<<<blocks, threads, 0, s>>>(static_cast<const uint8_t *>(src), type, n, dst);
    return cudaGetLastError();
}

cudaError_t launch_encproj_f32(const float * enc, int64_t frames, int De, const float * w,
                               const float * b, int J, float * out, cudaStream_t s) {
    if (frames <= 0) return cudaSuccess;
    dim3 grid((unsigned) ((frames + GB_M - 1) / GB_M), (unsigned) ((J + GB_N - 1) / GB_N));
    const bool vec = De % 4 == 0 && (reinterpret_cast<uintptr_t>(enc) & 15u) == 0 &&
                     (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
    if (vec) encproj_f32_kernel<true><<<grid, 256, 0, s>>>(enc, frames, De, w, b, J, out);
    else encproj_f32_kernel<false><<<grid, 256, 0, s>>>(enc, frames, De, w, b, J, out);
    return cudaGetLastError();
}

cudaError_t launch_scan(const int32_t * ust, int B, int field, int64_t * offsets, cudaStream_t s) {
    scan_counts_kernel<<<1, 1024, 0, s>>>(ust, B, field, offsets);
    return cudaGetLastError();
}

cudaError_t launch_gather(const int32_t * ust, int B, int field, const int32_t * src,
                          const int64_t * region, const int64_t * offsets, int32_t * dst,
                          cudaStream_t s) {
    if (B <= 0) return cudaSuccess;
    gather_kernel<<<B, 128, 0, s>>>(ust, field, src, region, offsets, dst);
    return cudaGetLastError();
}

cudaError_t launch_split_f16(const float * src, unsigned short * hi, unsigned short * lo, int64_t n,
                             cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    split_f16_kernel<<<(unsigned) ((n + 255) / 256), 256, 0, s>>>(src, reinterpret_cast<__half *>(hi),
                                                                reinterpret_cast<__half *>(lo), n);
    return cudaGetLastError();
}

cudaError_t launch_split_int16(const float * src, unsigned char * hi, unsigned char * lo, int64_t n,
                               cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    split_int16_kernel<<<(unsigned) ((n + 255) / 256), 256, 0, s>>>(src, reinterpret_cast<int8_t *>(hi), lo, n);
    return cudaGetLastError();
}

cudaError_t launch_stage_rows(const float * src, int n_rows, int H, int es, int rb, unsigned char * dst,
                              cudaStream_t s) {
    const int n = n_rows * H;
    if (n <= 0) return cudaSuccess;
    stage_rows_kernel<<<(n + 255) / 256, 256, 0, s>>>(src, n_rows, H, es, rb, dst);
    return cudaGetLastError();
}

// Copies of small host arrays staged in pinned host memory, read by the SMs over
// the bus (so they do not queue behind a large host-to-device copy in flight on
// the copy engines, as a prefetched batch's encoder copy is).
__global__ void copy_segments_kernel(HostSegments g) {
    const long long stride = (long long) gridDim.x * blockDim.x;
    for (int i = 0; i < g.n; ++i) {
        const unsigned * src = static_cast<const unsigned *>(g.seg[i].src);
        unsigned * dst = static_cast<unsigned *>(g.seg[i].dst);
        const long long words = (long long) (g.seg[i].bytes / 4);
        for (long long k = (long long) blockIdx.x * blockDim.x + threadIdx.x; k < words; k += stride) dst[k] = src[k];
    }
}

cudaError_t launch_copy_segments(const HostSegments & g, cudaStream_t s) {
    if (g.n <= 0) return cudaSuccess;
    unsigned long long words = 0;
    for (int i = 0; i < g.n; ++i) words += g.seg[i].bytes / 4;
    const unsigned blocks = (unsigned) std::min<unsigned long long>(64, (words + 255) / 256 + 1);
    copy_segments_kernel<<<blocks, 256, 0, s>>>(g);
    return cudaGetLastError();
}

cudaError_t launch_extract_field(const int32_t * ust, int B, int field, int32_t * dst,
                                 cudaStream_t s) {
    if (B <= 0) return cudaSuccess;
    extract_field_kernel<<<(B + 255) / 256, 256, 0, s>>>(ust, B, field, dst);
    return cudaGetLastError();
}

}  // namespace pk
