// pk_encproj.cu -- joint.enc projection of a whole batch of encoder frames on the
// 5th-generation tensor cores (tcgen05.mma, accumulator in tensor memory), weight
// tiles fed by TMA.
//
//   out[f][j] = b[j] + sum_k enc[f][k] * W[j][k]     (f < frames, j < J, k < De)
//
// The reference computes this per frame as an f32 gemv on dequantised weights
// (host_joint_step, parakeet_tdt.cpp:150-176; the GPU graph runs it once per
// window, build_enc_proj_graph, parakeet_tdt.cpp:433-483). To stay at f32-level
// accuracy on f16 tensor cores both operands are split into two f16 halves
// (x = x_hi + x_lo with x_hi = f16(x), x_lo = f16(x - x_hi)) and three products
// are accumulated in f32: A_hi.W_hi + A_lo.W_hi + A_hi.W_lo (the dropped
// A_lo.W_lo term is ~2^-22 relative). The weight halves are made once at load
// (q8_0 / f16 blocks -> exact f32 -> hi / lo); the encoder frames are split while
// they are staged into shared memory.
//
// Tile: 128 frames x 160 outputs per CTA, K in steps of 64 (one 128-byte
// swizzled row per operand row). Warp 4 issues every TMA load: the f32 frame
// tile (two-slot ring; rows past the last frame read as zero) and the f16 hi / lo
// weight tiles (two-slot operand ring). Warps 0-3 convert the f32 tile into the
// f16 hi / lo operand tiles (128B-swizzled, K-major) and run the epilogue; warp 5
// owns the tensor-memory allocation and issues the MMAs. Every wait is bounded.

#include "pk_umma.cuh"

#include <cuda_fp16.h>

namespace pk {
namespace {

constexpr int kEpM = 128;        // frames per CTA (UMMA M)
constexpr int kEpN = 160;        // outputs per CTA (UMMA N)
constexpr int kEpK = 64;         // K per pipeline stage (one 128-byte f16 row)
constexpr int kEpStages = 2;     // operand ring
constexpr int kEpFStages = 2;    // f32 frame-tile ring
constexpr int kEpThreads = 192;  // 6 warps
constexpr unsigned kTileA = kEpM * kEpK * 2;   // bytes of one f16 A tile (16 KB)
constexpr unsigned kTileB = kEpN * kEpK * 2;   // bytes of one f16 W tile (20 KB)
constexpr unsigned kStageBytes = 2 * kTileA + 2 * kTileB;
constexpr unsigned kTileF = kEpM * kEpK * 4;   // bytes of one f32 frame tile (32 KB)
constexpr unsigned kTmemCols = 256;             // >= kEpN, power of two

struct EpSmem {
    // tiles: [stage][A_hi, A_lo, W_hi, W_lo], each 1024-byte aligned
    unsigned long long full_a[kEpStages];
    unsigned long long full_w[kEpStages];
    unsigned long long empty[kEpStages];
    unsigned long long full_f[kEpFStages];
    unsigned long long empty_f[kEpFStages];
    unsigned long long done;
    unsigned tmem_base;
    int err;
};

__global__ void __launch_bounds__(kEpThreads, 1)
encproj_tc_kernel(const __grid_constant__ CUtensorMap emap,   // [frames][K] f32
                  long long frames, int K,
                  const __grid_constant__ CUtensorMap wmap,   // [2 * J][K] f16: rows 0..J-1 hi, J..2J-1 lo
                  int J, const float * __restrict__ bias, float * __restrict__ out,
                  long long timeout_ns, int * err_out) {
    extern __shared__ __align__(1024) unsigned char ep_raw[];
    // 1024-byte alignment of the tile area (the swizzle pattern is on absolute address bits)
    unsigned char * tiles = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(ep_raw) + 1023) & ~(uintptr_t) 1023);
    unsigned char * ftiles = tiles + kEpStages * kStageBytes;
    EpSmem & S = *reinterpret_cast<EpSmem *>(ftiles + kEpFStages * kTileF);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long m0 = (long long) blockIdx.y * kEpM;
    const int n0 = blockIdx.x * kEpN;
    const int nks = K / kEpK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kEpStages; ++s) {
            mbar_init(&S.full_a[s], 128);
            mbar_init(&S.full_w[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        for (int s = 0; s < kEpFStages; ++s) {
            mbar_init(&S.full_f[s], 1);
            mbar_init(&S.empty_f[s], 128);
        }
        mbar_init(&S.done, 1);
        S.err = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(&S.tmem_base)), "r"(kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tmem = S.tmem_base;

    if (warp < 4) {
        // ---- convert: f32 frame tile -> f16 hi / lo operand tiles, swizzled ----
        // warp w converts rows [32w, 32w + 32); each instruction covers two rows
        // (16 lanes x 4 floats = one 256-byte row each)
        const int sub = lane >> 4;           // row within the pair
        const int c4 = (lane & 15) * 4;      // first of this lane's 4 columns
        for (int ks = 0; ks < nks; ++ks) {
            const int s = ks % kEpStages, sf = ks % kEpFStages;
            const unsigned ph = (unsigned) (ks / kEpStages) & 1u, phf = (unsigned) (ks / kEpFStages) & 1u;
            if (!mbar_wait(&S.full_f[sf], phf, timeout_ns, &S.err)) break;
            if (!mbar_wait(&S.empty[s], ph ^ 1u, timeout_ns, &S.err)) break;
            const float * ft = reinterpret_cast<const float *>(ftiles + sf * kTileF);
            unsigned char * ahi = tiles + s * kStageBytes;
            unsigned char * alo = ahi + kTileA;
#pragma unroll 4
            for (int rp = 0; rp < 16; ++rp) {
                const int r = warp * 32 + rp * 2 + sub;
                const float4 v = *reinterpret_cast<const float4 *>(ft + r * kEpK + c4);
                const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y);
                const __half h2 = __float2half_rn(v.z), h3 = __float2half_rn(v.w);
                const __half l0 = __float2half_rn(v.x - __half2float(h0)), l1 = __float2half_rn(v.y - __half2float(h1));
                const __half l2 = __float2half_rn(v.z - __half2float(h2)), l3 = __float2half_rn(v.w - __half2float(h3));
                const unsigned off = (unsigned) r * 128u + ((((unsigned) c4 >> 3) ^ ((unsigned) r & 7u)) << 4) +
                                     ((unsigned) (c4 & 7) << 1);
                __half2 hp0 = __halves2half2(h0, h1), hp1 = __halves2half2(h2, h3);
                __half2 lp0 = __halves2half2(l0, l1), lp1 = __halves2half2(l2, l3);
                uint2 hv, lv;
                hv.x = *reinterpret_cast<unsigned *>(&hp0); hv.y = *reinterpret_cast<unsigned *>(&hp1);
                lv.x = *reinterpret_cast<unsigned *>(&lp0); lv.y = *reinterpret_cast<unsigned *>(&lp1);
                *reinterpret_cast<uint2 *>(ahi + off) = hv;
                *reinterpret_cast<uint2 *>(alo + off) = lv;
            }
            // the f32 slot may be refilled; the operand writes go to the async proxy
            mbar_arrive(&S.empty_f[sf]);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(&S.full_a[s]);
        }
    } else if (warp == 4) {
        // ---- every TMA load: f32 frame tiles and f16 weight tiles ----
        if (lane == 0) {
            for (int ks = 0; ks < nks; ++ks) {
                const int s = ks % kEpStages, sf = ks % kEpFStages;
                const unsigned ph = (unsigned) (ks / kEpStages) & 1u, phf = (unsigned) (ks / kEpFStages) & 1u;
                if (!mbar_wait(&S.empty_f[sf], phf ^ 1u, timeout_ns, &S.err)) break;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                             :: "r"(smem_u32(&S.full_f[sf])), "r"(kTileF) : "memory");
                tma_load_2d(ftiles + sf * kTileF, &emap, ks * kEpK, (int) m0, &S.full_f[sf]);
                if (!mbar_wait(&S.empty[s], ph ^ 1u, timeout_ns, &S.err)) break;
                unsigned char * whi = tiles + s * kStageBytes + 2 * kTileA;
                unsigned char * wlo = whi + kTileB;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                             :: "r"(smem_u32(&S.full_w[s])), "r"(2u * kTileB) : "memory");
                tma_load_2d(whi, &wmap, ks * kEpK, n0, &S.full_w[s]);
                tma_load_2d(wlo, &wmap, ks * kEpK, J + n0, &S.full_w[s]);
            }
        }
    } else {
        // ---- MMA issuer ----
        if (lane == 0) {
            constexpr unsigned idesc = umma_idesc_f16(kEpM, kEpN);
            for (int ks = 0; ks < nks; ++ks) {
                const int s = ks % kEpStages;
                const unsigned ph = (unsigned) (ks / kEpStages) & 1u;
                if (!mbar_wait(&S.full_a[s], ph, timeout_ns, &S.err)) break;
                if (!mbar_wait(&S.full_w[s], ph, timeout_ns, &S.err)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const unsigned base = smem_u32(tiles + s * kStageBytes);
                const unsigned ahi = base, alo = base + kTileA, whi = base + 2 * kTileA, wlo = whi + kTileB;
#pragma unroll
                for (int k16 = 0; k16 < kEpK / 16; ++k16) {
                    const unsigned ko = (unsigned) k16 * 32u;   // 16 f16 = 32 bytes along the swizzled row
                    umma_f16(tmem, umma_desc_sw128(ahi + ko), umma_desc_sw128(whi + ko), idesc, (ks | k16) ? 1u : 0u);
                    umma_f16(tmem, umma_desc_sw128(alo + ko), umma_desc_sw128(whi + ko), idesc, 1u);
                    umma_f16(tmem, umma_desc_sw128(ahi + ko), umma_desc_sw128(wlo + ko), idesc, 1u);
                }
                umma_commit(&S.empty[s]);   // stage free once these MMAs have read it
            }
            umma_commit(&S.done);           // accumulator complete
        }
    }

    // ---- epilogue: TMEM -> registers -> +bias -> global (warps 0-3, row = TMEM lane) ----
    if (warp < 4) {
        const bool ok = mbar_wait(&S.done, 0u, timeout_ns, &S.err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (ok) {
            const int r = warp * 32 + lane;
            const long long f = m0 + r;
#pragma unroll 1
            for (int c0 = 0; c0 < kEpN; c0 += 16) {
                unsigned v[16];
                const unsigned taddr = tmem + ((unsigned) (warp * 32) << 16) + (unsigned) c0;
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                             "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                             : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                               "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
                               "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                             : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (f < frames) {
                    float * o = out + f * J + n0 + c0;
#pragma unroll
                    for (int q = 0; q < 16; q += 4) {
                        float4 w;
                        w.x = __ldg(bias + n0 + c0 + q + 0) + __uint_as_float(v[q + 0]);
                        w.y = __ldg(bias + n0 + c0 + q + 1) + __uint_as_float(v[q + 1]);
                        w.z = __ldg(bias + n0 + c0 + q + 2) + __uint_as_float(v[q + 2]);
                        w.w = __ldg(bias + n0 + c0 + q + 3) + __uint_as_float(v[q + 3]);
                        *reinterpret_cast<float4 *>(o + q) = w;
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 5) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(kTmemCols) : "memory");
    }
    if (threadIdx.x == 0 && S.err != 0) atomicExch(err_out, 1);
}

// w (f32, [J][K]) -> [2J][K] f16: rows 0..J-1 = f16(w), rows J..2J-1 = f16(w - f16(w)).
__global__ void split_weight_kernel(const float * __restrict__ w, long long n, __half * __restrict__ out) {
    const long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float x = w[i];
    const __half h = __float2half_rn(x);
    out[i] = h;
    out[n + i] = __float2half_rn(x - __half2float(h));
}

}  // namespace

size_t encproj_tc_smem_bytes() {
    return 1024 + (size_t) kEpStages * kStageBytes + (size_t) kEpFStages * kTileF + sizeof(EpSmem);
}

bool encproj_tc_supported(int K, int J) { return K > 0 && K % kEpK == 0 && J > 0 && J % kEpN == 0; }

using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
    static EncodeFn fn = nullptr;
    if (fn == nullptr) {
        void * p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeFn>(p);
    }
    return fn;
}

// 2-D row-major tensor map: rows x cols of `type`, box box_rows x box_cols.
cudaError_t encode_2d(void * map, CUtensorMapDataType type, size_t esize, const void * base, long long rows,
                      long long cols, int box_rows, int box_cols, CUtensorMapSwizzle swz) {
    EncodeFn fn = encode_fn();
    if (fn == nullptr) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t) cols, (cuuint64_t) rows};
    const cuuint64_t strides[1] = {(cuuint64_t) cols * esize};
    const cuuint32_t box[2] = {(cuuint32_t) box_cols, (cuuint32_t) box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(reinterpret_cast<CUtensorMap *>(map), type, 2, const_cast<void *>(base), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t encproj_tc_prepare(const float * w, int J, int K, unsigned short * w16, void * tmap_out, cudaStream_t s) {
    const long long n = (long long) J * K;
    split_weight_kernel<<<(unsigned) ((n + 255) / 256), 256, 0, s>>>(w, n, reinterpret_cast<__half *>(w16));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return encode_2d(tmap_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w16, 2LL * J, K, kEpN, kEpK,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

cudaError_t encproj_tc_configure() {
    return cudaFuncSetAttribute(encproj_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int) encproj_tc_smem_bytes());
}

cudaError_t launch_encproj_tc(const float * enc, long long frames, int K, const void * tmap, int J,
                              const float * bias, float * out, long long timeout_ns, int * err, cudaStream_t s) {
    if (frames <= 0) return cudaSuccess;
    if ((reinterpret_cast<uintptr_t>(enc) & 15u) != 0) return cudaErrorMisalignedAddress;
    alignas(64) CUtensorMap emap;
    cudaError_t e = encode_2d(&emap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, enc, frames, K, kEpM, kEpK,
                              CU_TENSOR_MAP_SWIZZLE_NONE);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned) (J / kEpN), (unsigned) ((frames + kEpM - 1) / kEpM));
    encproj_tc_kernel<<<grid, kEpThreads, encproj_tc_smem_bytes(), s>>>(
        emap, frames, K, *reinterpret_cast<const CUtensorMap *>(tmap), J, bias, out, timeout_ns, err);
    return cudaGetLastError();
}

}  // namespace pk
