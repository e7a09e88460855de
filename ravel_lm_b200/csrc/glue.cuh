// glue.cuh -- the elementwise and row-norm work a memory layer does around the
// operator (ravel_lm/model.py:388 gate_residual, model.py:35-36 RMSNorm).
//
//   k_gate_res_fwd  out = x + sigmoid(gate) * fused, one pass over three inputs.
//                   The stock model's CUDA path runs this as three torch kernels
//                   (sigmoid, mul, add: triton_block.py:383-387 with its Triton
//                   glue switched off); the arithmetic and rounding order are the
//                   same as those kernels', so results are equal bit for bit.
//   k_gate_res_bwd  d gate = ((gy * fused) * (1 - s)) * s, d fused = gy * s with
//                   s = sigmoid(gate) recomputed; the order of torch's mul and
//                   sigmoid backward formulas, one pass.
//   k_rms_fwd       y = x * rsqrt(mean(x^2) + eps) * g per row, one warp per row;
//                   keeps rstd per row for the backward.
//   k_rms_bwd       dx = rstd * (gy*g) - rstd^3 / K * dot(gy*g, x) * x per row;
//                   dg = sum over rows of gy * x * rstd, as per-block partial rows
//                   (a fixed row -> block mapping, summed in a fixed order by
//                   k_rms_dg_reduce): deterministic, no atomics.
// Every kernel is HBM-bound: it reads and writes each element once.
#pragma once

#include "common.cuh"

namespace ravel {

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// 1 / (1 + exp(-x)) in float, the formula of torch's sigmoid kernel for float.
__device__ __forceinline__ float sigmoid_f(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

// Vectors of 16 bytes when every pointer and the element count allow, else scalars.
template <typename T>
__global__ void __launch_bounds__(256) k_gate_res_fwd(const T* __restrict__ x, const T* __restrict__ gate,
                                                      const T* __restrict__ fused, T* __restrict__ out, int64_t n,
                                                      int vec) {
    constexpr int EPV = 16 / sizeof(T);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (vec) {
        for (int64_t v = i0; v < n / EPV; v += stride) {
            const uint4 xa = ld_nc_v4(x + v * EPV), ga = ld_nc_v4(gate + v * EPV), fa = ld_nc_v4(fused + v * EPV);
            const T* xs = reinterpret_cast<const T*>(&xa);
            const T* gs = reinterpret_cast<const T*>(&ga);
            const T* fs = reinterpret_cast<const T*>(&fa);
            uint4 o;
            T* os = reinterpret_cast<T*>(&o);
#pragma unroll
            for (int e = 0; e < EPV; ++e) {
                // torch: sigmoid (rounded to T), mul (rounded to T), add (rounded to T)
                const float s = to_f(from_f<T>(sigmoid_f(to_f(gs[e]))));
                const float m = to_f(from_f<T>(__fmul_rn(s, to_f(fs[e]))));
                os[e] = from_f<T>(__fadd_rn(to_f(xs[e]), m));
            }
            *reinterpret_cast<uint4*>(out + v * EPV) = o;
        }
        return;
    }
    for (int64_t i = i0; i < n; i += stride) {
        const float s = to_f(from_f<T>(sigmoid_f(to_f(gate[i]))));
        const float m = to_f(from_f<T>(__fmul_rn(s, to_f(fused[i]))));
        out[i] = from_f<T>(__fadd_rn(to_f(x[i]), m));
    }
}

template <typename T>
__device__ __forceinline__ void gate_res_bwd_one(T gy, T g, T f, T& dg, T& df) {
    const float s = to_f(from_f<T>(sigmoid_f(to_f(g))));
    const float gyf = to_f(gy);
    // mul backward: d s = gy * fused, d fused = gy * s; sigmoid backward: (d s * (1 - s)) * s
    const float ds = to_f(from_f<T>(__fmul_rn(gyf, to_f(f))));
    const float oms = to_f(from_f<T>(__fsub_rn(1.0f, s)));  // 16-bit types round every step, as torch does
    dg = from_f<T>(__fmul_rn(to_f(from_f<T>(__fmul_rn(ds, oms))), s));
    df = from_f<T>(__fmul_rn(gyf, s));
}

template <typename T>
__global__ void __launch_bounds__(256) k_gate_res_bwd(const T* __restrict__ gate, const T* __restrict__ fused,
                                                      const T* __restrict__ gy, T* __restrict__ dgate,
                                                      T* __restrict__ dfused, int64_t n, int vec) {
    constexpr int EPV = 16 / sizeof(T);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (vec) {
        for (int64_t v = i0; v < n / EPV; v += stride) {
            const uint4 ga = ld_nc_v4(gate + v * EPV), fa = ld_nc_v4(fused + v * EPV), ya = ld_nc_v4(gy + v * EPV);
            const T* gs = reinterpret_cast<const T*>(&ga);
            const T* fs = reinterpret_cast<const T*>(&fa);
            const T* ys = reinterpret_cast<const T*>(&ya);
            uint4 og, of;
            T* ogs = reinterpret_cast<T*>(&og);
            T* ofs = reinterpret_cast<T*>(&of);
#pragma unroll
            for (int e = 0; e < EPV; ++e) gate_res_bwd_one<T>(ys[e], gs[e], fs[e], ogs[e], ofs[e]);
            *reinterpret_cast<uint4*>(dgate + v * EPV) = og;
            *reinterpret_cast<uint4*>(dfused + v * EPV) = of;
        }
        return;
    }
    for (int64_t i = i0; i < n; i += stride) gate_res_bwd_one<T>(gy[i], gate[i], fused[i], dgate[i], dfused[i]);
}

// ------------------------------------------------------------------ RMSNorm
// One warp per row; rows are taken in a grid-stride order that depends only on
// M and the grid, so the backward's per-block dg partials are reproducible.
template <typename T>
__global__ void __launch_bounds__(256) k_rms_fwd(const T* __restrict__ x, const T* __restrict__ g,
                                                 T* __restrict__ y, float* __restrict__ rstd, int64_t M, int K,
                                                 float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t w0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t row = w0; row < M; row += nw) {
        const T* xr = x + row * K;
        float ss = 0.0f;
        for (int j = lane; j < K; j += 32) {
            const float v = to_f(xr[j]);
            ss = fmaf(v, v, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float r = rsqrtf(ss / static_cast<float>(K) + eps);
        T* yr = y + row * K;
        for (int j = lane; j < K; j += 32) yr[j] = from_f<T>(to_f(xr[j]) * r * to_f(g[j]));
        if (lane == 0) rstd[row] = r;
    }
}

// dx per row; dg partial per block: part[block][K] (float), summed over the
// block's warps in warp order after every row is done.
template <typename T>
__global__ void __launch_bounds__(256) k_rms_bwd(const T* __restrict__ x, const T* __restrict__ g,
                                                 const T* __restrict__ gy, const float* __restrict__ rstd,
                                                 T* __restrict__ dx, float* __restrict__ part, int64_t M, int K) {
    extern __shared__ float wpart[];  // [warps][K]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwb = blockDim.x >> 5;
    float* mine = wpart + static_cast<int64_t>(warp) * K;
    for (int j = lane; j < K; j += 32) mine[j] = 0.0f;
    const int64_t w0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t row = w0; row < M; row += nw) {
        const T* xr = x + row * K;
        const T* gr = gy + row * K;
        const float r = rstd[row];
        float dot = 0.0f;
        for (int j = lane; j < K; j += 32) dot = fmaf(to_f(gr[j]) * to_f(g[j]), to_f(xr[j]), dot);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float c = r * r * r / static_cast<float>(K) * dot;
        T* dr = dx + row * K;
        for (int j = lane; j < K; j += 32) {
            const float xv = to_f(xr[j]), gv = to_f(gr[j]);
            dr[j] = from_f<T>(r * gv * to_f(g[j]) - c * xv);
            mine[j] += gv * xv * r;
        }
    }
    __syncthreads();
    for (int j = threadIdx.x; j < K; j += blockDim.x) {
        float s = 0.0f;
        for (int w = 0; w < nwb; ++w) s += wpart[static_cast<int64_t>(w) * K + j];
        part[static_cast<int64_t>(blockIdx.x) * K + j] = s;
    }
}

template <typename T>
__global__ void __launch_bounds__(256) k_rms_dg_reduce(const float* __restrict__ part, int nblocks, int K,
                                                       T* __restrict__ dg) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= K) return;
    float s = 0.0f;
    for (int b = 0; b < nblocks; ++b) s += part[static_cast<int64_t>(b) * K + j];
    dg[j] = from_f<T>(s);
}

}  // namespace ravel
