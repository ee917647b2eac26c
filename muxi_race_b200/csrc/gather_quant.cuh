// gather_quant.cuh — row movement and int8 quantisation around the grouped GEMMs.
//
//   gather_rows       xs[route_slot[r]] = x[r / topk] for every routed row r (the stacked,
//                     expert-grouped layout the reference receives pre-built as
//                     stacked_expert_tokens), and zero the token-major output that the Stage2
//                     epilogue accumulates into. One warp per row, 16-byte vectors.
//   gather_rows_q8    the same gather with per-token symmetric int8 quantisation fused in:
//                     scale = amax(|x[t]|) / 127, q = clamp(round_half_away(x / scale), +-127).
//   quantize_rows_q8  per-row amax int8 (or fp8) quantisation of a [rows, K] 16-bit matrix
//                     (weights offline: one scale per output row; the Stage1 intermediate online).
// The rounding and clamp follow the reference's int8 experiment
// (xpuoj_data/submission_v322_int8_v2.py:186-203): amax/127 scale, round half away from zero,
// clamp to [-127, 127]. The fp8 kind (Q8 = kQF8) uses the same per-row scheme with the e4m3
// range: scale = amax / 448, q = e4m3(x * (448 / amax)) rounded to nearest even and saturated to
// +-448 by CUDA's conversion intrinsic.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace moe {

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f<T>(e[i]);
}

__device__ __forceinline__ int8_t q8(float v, float inv_scale) {
  float q = roundf(v * inv_scale);
  q = fminf(fmaxf(q, -127.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(q));
}

// Per-kind encoding of one scaled value (inv = kMax / amax) into its byte.
template <int Q8> struct QuantKind;
template <> struct QuantKind<kQI8> {
  static constexpr float kMax = 127.0f;
  static __device__ __forceinline__ uint32_t enc(float v, float inv) { return static_cast<uint8_t>(q8(v, inv)); }
};
template <> struct QuantKind<kQF8> {
  static constexpr float kMax = 448.0f;
  static __device__ __forceinline__ uint32_t enc(float v, float inv) {
    return static_cast<uint32_t>(__nv_cvt_float_to_fp8(v * inv, __NV_SATFINITE, __NV_E4M3));
  }
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// rows_zero rows of `zero_out` (row length zero_ld elements of 2 bytes) are cleared after the
// gather work items; zero_f32[0..n_zero_f32) is cleared too (Stage1 int8 row amax).
template <typename T>
__global__ void gather_rows_kernel(const T* __restrict__ x, const int32_t* __restrict__ route_slot, int R, int topk,
                                   int H, T* __restrict__ xs, T* __restrict__ zero_out, int zero_rows,
                                   float* __restrict__ zero_f32, int n_zero_f32) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const int vecs = H / 8;
  for (long long item = warp_id; item < static_cast<long long>(R) + zero_rows; item += n_warps) {
    if (item < R) {
      const int slot = route_slot[item];
      if (slot < 0) continue;
      const uint4* src = reinterpret_cast<const uint4*>(x + (item / topk) * static_cast<size_t>(H));
      uint4* dst = reinterpret_cast<uint4*>(xs + static_cast<size_t>(slot) * H);
      for (int v = lane; v < vecs; v += 32) dst[v] = __ldg(src + v);
    } else {
      uint4* dst = reinterpret_cast<uint4*>(zero_out + (item - R) * static_cast<size_t>(H));
      for (int v = lane; v < vecs; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
    }
  }
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (long long i = tid; i < n_zero_f32; i += static_cast<long long>(gridDim.x) * blockDim.x) zero_f32[i] = 0.0f;
}

template <typename T, int Q8 = kQI8>
__global__ void gather_rows_q8_kernel(const T* __restrict__ x, const int32_t* __restrict__ route_slot, int R, int topk,
                                      int H, int8_t* __restrict__ xq, float* __restrict__ xscale,
                                      T* __restrict__ zero_out, int zero_rows, float* __restrict__ zero_f32,
                                      int n_zero_f32) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const int vecs = H / 8;
  for (long long item = warp_id; item < static_cast<long long>(R) + zero_rows; item += n_warps) {
    if (item < R) {
      const int slot = route_slot[item];
      if (slot < 0) continue;
      const uint4* src = reinterpret_cast<const uint4*>(x + (item / topk) * static_cast<size_t>(H));
      float amax = 0.0f;
      for (int v = lane; v < vecs; v += 32) {
        float f[8];
        unpack8<T>(__ldg(src + v), f);
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
      }
      amax = warp_max(amax);
      const float inv = amax > 0.0f ? QuantKind<Q8>::kMax / amax : 0.0f;
      uint2* dst = reinterpret_cast<uint2*>(xq + static_cast<size_t>(slot) * H);
      for (int v = lane; v < vecs; v += 32) {
        float f[8];
        unpack8<T>(__ldg(src + v), f);
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) w0 |= QuantKind<Q8>::enc(f[i], inv) << (8 * i);
#pragma unroll
        for (int i = 0; i < 4; ++i) w1 |= QuantKind<Q8>::enc(f[4 + i], inv) << (8 * i);
        dst[v] = make_uint2(w0, w1);
      }
      if (lane == 0) xscale[slot] = amax / QuantKind<Q8>::kMax;
    } else {
      uint4* dst = reinterpret_cast<uint4*>(zero_out + (item - R) * static_cast<size_t>(H));
      for (int v = lane; v < vecs; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
    }
  }
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (long long i = tid; i < n_zero_f32; i += static_cast<long long>(gridDim.x) * blockDim.x) zero_f32[i] = 0.0f;
}

// Quantise rows [0, rows) of a [rows, K] matrix. If `row_amax` is given the per-row amax is
// taken from it (Stage1 computed it in its epilogue); otherwise it is computed here.
// `nrows_dev` (optional) bounds the rows on the device (padded row count of the routing).
template <typename T, int Q8 = kQI8>
__global__ void quantize_rows_q8_kernel(const T* __restrict__ w, long long rows, int K, const int* __restrict__ nrows_dev,
                                        const float* __restrict__ row_amax, int8_t* __restrict__ q,
                                        float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  if (nrows_dev) rows = min(rows, static_cast<long long>(*nrows_dev));
  const int vecs = K / 8;
  for (long long r = warp_id; r < rows; r += n_warps) {
    const uint4* src = reinterpret_cast<const uint4*>(w + r * K);
    float amax;
    if (row_amax) {
      amax = row_amax[r];
    } else {
      amax = 0.0f;
      for (int v = lane; v < vecs; v += 32) {
        float f[8];
        unpack8<T>(__ldg(src + v), f);
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
      }
      amax = warp_max(amax);
    }
    const float inv = amax > 0.0f ? QuantKind<Q8>::kMax / amax : 0.0f;
    uint2* dst = reinterpret_cast<uint2*>(q + r * K);
    for (int v = lane; v < vecs; v += 32) {
      float f[8];
      unpack8<T>(__ldg(src + v), f);
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) w0 |= QuantKind<Q8>::enc(f[i], inv) << (8 * i);
#pragma unroll
      for (int i = 0; i < 4; ++i) w1 |= QuantKind<Q8>::enc(f[4 + i], inv) << (8 * i);
      dst[v] = make_uint2(w0, w1);
    }
    if (lane == 0) scale[r] = amax / QuantKind<Q8>::kMax;
  }
}

}  // namespace moe
