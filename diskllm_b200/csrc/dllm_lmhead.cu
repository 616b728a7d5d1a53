// dllm_lmhead.cu -- the step before the sampler: final RMSNorm, logits matvec, optional softcap
// (DiskLLM src/core/context.c:854-876), for unquantised output weights (f32, f16, bf16).
//
//   norm    src/rmsnorm.c:4-27   ss = sum of x^2 in double, / n, + eps; scale = (float)(1/sqrt(ss));
//                                then in fp32, as the reference compiles at -O3 -ffast-math:
//                                x * scale, (x * scale) * (w + 1), or (x * w) * scale
//   matvec  src/matvec.c:251-366 per output row, sum in double of (double)w * (double)x, then
//                                rounded to float once
//   softcap context.c:873-876    logit = cap * tanhf(logit / cap) when cap > 0
//
// The matvec reads each weight once (vocab x hidden elements, 1 GB for 128256 x 4096 bf16) and
// is HBM-bound for decode batches: one warp per output row streams the row with 16-byte loads and
// keeps one double accumulator per batch row (up to LMH_MAXB); the partial sums are combined by a
// shuffle tree, so the order of the double additions differs from the reference's sequential loop
// (relative 1e-16: the rounded float agrees except at ties).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "dllm_internal.h"

namespace dllm {
namespace {

constexpr int LMH_MAXB = 8;     // batch rows per launch of the matvec
constexpr int LMH_THREADS = 256;

// one CTA per batch row: the normalised row in fp32 (as the reference's rmsnorm_ext writes it)
__global__ void rmsnorm_rows_kernel(const float *x, const float *w, int hidden, float eps, int add_one, float *out) {
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
    const float *xr = x + (size_t)b * hidden;
    __shared__ double part[32];
    double ss = 0.0;
    for (int i = tid; i < hidden; i += blockDim.x) ss += (double)xr[i] * (double)xr[i];
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) part[wid] = ss;
    __syncthreads();
    double tot = 0.0;
    for (int i = 0; i < nw; i++) tot += part[i];
    tot = tot / (double)hidden + (double)eps;
    const float scale = __double2float_rn(1.0 / sqrt(tot));
    float *orow = out + (size_t)b * hidden;
    for (int i = tid; i < hidden; i += blockDim.x) {
        orow[i] = !w ? __fmul_rn(xr[i], scale)
                     : (add_one ? __fmul_rn(__fmul_rn(xr[i], scale), __fadd_rn(w[i], 1.0f))
                                : __fmul_rn(__fmul_rn(xr[i], w[i]), scale));
    }
}

template <int WT>
__device__ __forceinline__ void load8(const void *row, int j, float (&f)[8]) {
    if (WT == DLLM_DTYPE_F32) {
        const float4 a = *reinterpret_cast<const float4 *>((const float *)row + j);
        const float4 c = *reinterpret_cast<const float4 *>((const float *)row + j + 4);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = c.x; f[5] = c.y; f[6] = c.z; f[7] = c.w;
    } else {
        const uint4 raw = *reinterpret_cast<const uint4 *>((const unsigned short *)row + j);
        const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if (WT == DLLM_DTYPE_BF16) {
                f[2 * k] = __uint_as_float(u[k] << 16);
                f[2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
            } else {
                f[2 * k] = __half2float(__ushort_as_half((unsigned short)(u[k] & 0xffffu)));
                f[2 * k + 1] = __half2float(__ushort_as_half((unsigned short)(u[k] >> 16)));
            }
        }
    }
}

// one warp per LMH_RV output rows (grid-stride over groups of rows).  Lane l of a warp reads
// weights 256 m + 8 l .. + 7 of each of its rows with one 16-byte load; the normalised batch rows
// sit in shared memory as doubles in the matching interleaved order -- element 256 m + 8 l + k at
// 256 m + 32 k + l -- so the lanes' reads of one k hit 32 consecutive doubles (no bank conflicts),
// and each double read from shared memory feeds LMH_RV fused multiply-adds (the reads, not the
// weight stream, bound a warp that covers one row at a time once the batch has several rows).
__device__ __forceinline__ int lmh_perm(int j) { return (j & ~255) + (j & 7) * 32 + ((j >> 3) & 31); }

constexpr int LMH_RV = 4;

template <int WT, int NB>
__global__ void __launch_bounds__(LMH_THREADS) lmhead_matvec_kernel(const float *hn, const void *w, int hidden, int hp,
                                                                    int vocab, float softcap, float *logits) {
    extern __shared__ __align__(16) double xs[];  // [NB][hp]
    const int tid = threadIdx.x, lane = tid & 31;
    for (int i = tid; i < NB * hidden; i += blockDim.x) {
        const int b = i / hidden, j = i - b * hidden;
        xs[b * hp + lmh_perm(j)] = (double)hn[i];
    }
    __syncthreads();
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const size_t esz = WT == DLLM_DTYPE_F32 ? 4 : 2;
    for (int row0 = ((blockIdx.x * blockDim.x + tid) >> 5) * LMH_RV; row0 < vocab; row0 += warps * LMH_RV) {
        const unsigned char *wrow[LMH_RV];
#pragma unroll
        for (int r = 0; r < LMH_RV; r++) {  // rows past the vocabulary re-read the last row; not stored
            const int row = row0 + r < vocab ? row0 + r : vocab - 1;
            wrow[r] = (const unsigned char *)w + (size_t)row * hidden * esz;
        }
        double acc[LMH_RV][NB];
#pragma unroll
        for (int r = 0; r < LMH_RV; r++)
#pragma unroll
            for (int b = 0; b < NB; b++) acc[r][b] = 0.0;
        for (int base = 0; base < hidden; base += 256) {
            const int j = base + 8 * lane;
            if (j < hidden) {  // hidden is a multiple of 8
                float f[LMH_RV][8];
#pragma unroll
                for (int r = 0; r < LMH_RV; r++) load8<WT>(wrow[r], j, f[r]);
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const int xi = base + 32 * k + lane;
#pragma unroll
                    for (int b = 0; b < NB; b++) {
                        const double xv = xs[b * hp + xi];
#pragma unroll
                        for (int r = 0; r < LMH_RV; r++) acc[r][b] = fma((double)f[r][k], xv, acc[r][b]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < LMH_RV; r++) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
#pragma unroll
                for (int o = 16; o; o >>= 1) acc[r][b] += __shfl_xor_sync(0xffffffffu, acc[r][b], o);
            }
            if (lane < NB && row0 + r < vocab) {
                double v = acc[r][0];
#pragma unroll
                for (int b = 1; b < NB; b++)
                    if (lane == b) v = acc[r][b];
                float lg = __double2float_rn(v);
                if (softcap > 0.0f) lg = __fmul_rn(softcap, tanhf(__fdiv_rn(lg, softcap)));
                logits[(size_t)lane * vocab + row0 + r] = lg;
            }
        }
    }
}

template <int WT, int NB>
cudaError_t launch_matvec(const float *hn, const void *w, int hidden, int vocab, float softcap, float *logits,
                          cudaStream_t stream) {
    const int hp = (hidden + 255) & ~255;
    const size_t smem = (size_t)NB * hp * sizeof(double);
    cudaError_t e = cudaFuncSetAttribute((const void *)lmhead_matvec_kernel<WT, NB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lmhead_matvec_kernel<WT, NB>, LMH_THREADS, smem);
    const int rows_per_block = LMH_THREADS / 32 * LMH_RV;
    int grid = sms * (per_sm > 0 ? per_sm : 1);
    const int need = (vocab + rows_per_block - 1) / rows_per_block;
    if (grid > need) grid = need;
    lmhead_matvec_kernel<WT, NB><<<grid, LMH_THREADS, smem, stream>>>(hn, w, hidden, hp, vocab, softcap, logits);
    return cudaGetLastError();
}

template <int WT>
cudaError_t dispatch_nb(int nb, const float *hn, const void *w, int hidden, int vocab, float softcap, float *logits,
                        cudaStream_t s) {
    switch (nb) {
        case 1: return launch_matvec<WT, 1>(hn, w, hidden, vocab, softcap, logits, s);
        case 2: return launch_matvec<WT, 2>(hn, w, hidden, vocab, softcap, logits, s);
        case 3: return launch_matvec<WT, 3>(hn, w, hidden, vocab, softcap, logits, s);
        case 4: return launch_matvec<WT, 4>(hn, w, hidden, vocab, softcap, logits, s);
        case 5: return launch_matvec<WT, 5>(hn, w, hidden, vocab, softcap, logits, s);
        case 6: return launch_matvec<WT, 6>(hn, w, hidden, vocab, softcap, logits, s);
        case 7: return launch_matvec<WT, 7>(hn, w, hidden, vocab, softcap, logits, s);
        default: return launch_matvec<WT, 8>(hn, w, hidden, vocab, softcap, logits, s);
    }
}

}  // namespace

// batch rows one launch can hold in shared memory (doubles, padded to 256)
int lmh_max_rows(int hidden) {
    const int hp = (hidden + 255) & ~255;
    const int n = (int)((200 * 1024) / ((size_t)hp * sizeof(double)));
    return n < 1 ? 0 : (n > LMH_MAXB ? LMH_MAXB : n);
}

dllm_status launch_lmhead(int rows, int hidden, int vocab, const float *h, const float *norm_w, float eps, int add_one,
                          const void *w, int w_dtype, float softcap, float *logits, float *scratch,
                          cudaStream_t stream) {
    if (rows == 0) return DLLM_OK;
    rmsnorm_rows_kernel<<<rows, 256, 0, stream>>>(h, norm_w, hidden, eps, add_one, scratch);
    if (cudaGetLastError() != cudaSuccess) return DLLM_ERR_CUDA;
    const int maxb = lmh_max_rows(hidden);
    if (maxb < 1) return DLLM_ERR_UNSUPPORTED;
    for (int r0 = 0; r0 < rows; r0 += maxb) {
        const int nb = rows - r0 < maxb ? rows - r0 : maxb;
        const float *hn = scratch + (size_t)r0 * hidden;
        float *out = logits + (size_t)r0 * vocab;
        cudaError_t e;
        if (w_dtype == DLLM_DTYPE_F32) e = dispatch_nb<DLLM_DTYPE_F32>(nb, hn, w, hidden, vocab, softcap, out, stream);
        else if (w_dtype == DLLM_DTYPE_BF16) e = dispatch_nb<DLLM_DTYPE_BF16>(nb, hn, w, hidden, vocab, softcap, out, stream);
        else e = dispatch_nb<DLLM_DTYPE_F16>(nb, hn, w, hidden, vocab, softcap, out, stream);
        if (e != cudaSuccess) return DLLM_ERR_CUDA;
    }
    return DLLM_OK;
}


}  // namespace dllm
