// ep_kernels.cuh — expert-parallel dispatch and combine around the NCCL all-to-all exchanges.
//
// Experts are owned by ranks (expert_rank[e], expert_local[e] = index among that rank's experts).
// A token is sent once to every rank that owns at least one of its top-k experts ("pairs" =
// (token, rank)); it travels with its k expert ids rewritten to the destination's local ids
// (-1 for experts owned elsewhere) and its k routing weights, so the destination runs the
// ordinary fused MoE on the received rows and the top-k combine of its local routes happens in
// that fused MoE's Stage2 epilogue. The partial outputs come back by the reverse all-to-all and
// are summed per token in a fixed rank order (deterministic given the partials).
//
// Send order = pairs sorted by destination rank, tokens ascending inside a rank: built with the
// routing alignment (route_align.cuh) over T*W pair keys with E = W and block size 1.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace moe {

// keys[t*W + r] = r if token t routes to an expert owned by rank r, else -1.
template <typename IdT>
__global__ void ep_pair_keys_kernel(const IdT* __restrict__ ids, int T, int topk, const int32_t* __restrict__ expert_rank,
                                    int E, int W, int32_t* __restrict__ keys) {
  const long long n = static_cast<long long>(T) * W;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / W), r = static_cast<int>(i % W);
    bool hit = false;
    for (int j = 0; j < topk; ++j) {
      const long long e = static_cast<long long>(ids[static_cast<long long>(t) * topk + j]);
      if (e >= 0 && e < E && expert_rank[e] == r) hit = true;
    }
    keys[i] = hit ? r : -1;
  }
}

// Pack send row p (< meta[2]) from pair v = send_pairs[p]: the token row, its k local expert ids
// for the destination (or -1) and its k weights as fp32. One warp per row.
template <typename T, typename IdT>
__global__ void ep_pack_kernel(const T* __restrict__ x, const IdT* __restrict__ ids, const void* __restrict__ w, int w_dtype,
                               const int32_t* __restrict__ expert_rank, const int32_t* __restrict__ expert_local, int E,
                               const int32_t* __restrict__ send_pairs, const int32_t* __restrict__ meta, int H,
                               int topk, int W, T* __restrict__ send_x, int32_t* __restrict__ send_ids,
                               float* __restrict__ send_w) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const long long n_send = meta[2];
  const int vecs = H / 8;
  for (long long p = warp_id; p < n_send; p += n_warps) {
    const int v = send_pairs[p];
    const int t = v / W, r = v % W;
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H);
    uint4* dst = reinterpret_cast<uint4*>(send_x + static_cast<size_t>(p) * H);
    for (int c = lane; c < vecs; c += 32) dst[c] = __ldg(src + c);
    for (int j = lane; j < topk; j += 32) {
      const long long e = static_cast<long long>(ids[static_cast<long long>(t) * topk + j]);
      const bool mine = e >= 0 && e < E && expert_rank[e] == r;
      send_ids[p * topk + j] = mine ? expert_local[e] : -1;
      const long long wi = static_cast<long long>(t) * topk + j;
      float wv;
      if (w_dtype == 0)
        wv = reinterpret_cast<const float*>(w)[wi];
      else if (w_dtype == 1)
        wv = __half2float(reinterpret_cast<const __half*>(w)[wi]);
      else
        wv = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[wi]);
      send_w[p * topk + j] = wv;
    }
  }
}

// out[t] = sum over ranks r (ascending) of y[pair_slot[t*W + r]] (fp32 sum, one rounding).
template <typename T>
__global__ void ep_combine_kernel(const T* __restrict__ y, const int32_t* __restrict__ pair_slot, int n_tokens, int H, int W,
                                  T* __restrict__ out);

template <>
__global__ void ep_combine_kernel<__half>(const __half* __restrict__ y, const int32_t* __restrict__ pair_slot, int n_tokens,
                                          int H, int W, __half* __restrict__ out) {
  const long long n = static_cast<long long>(n_tokens) * (H / 2);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / (H / 2));
    const int c2 = static_cast<int>(i % (H / 2));
    float a = 0.f, b = 0.f;
    for (int r = 0; r < W; ++r) {
      const int s = pair_slot[static_cast<long long>(t) * W + r];
      if (s >= 0) {
        const float2 f = __half22float2(reinterpret_cast<const __half2*>(y + static_cast<size_t>(s) * H)[c2]);
        a += f.x;
        b += f.y;
      }
    }
    reinterpret_cast<__half2*>(out + static_cast<size_t>(t) * H)[c2] = __floats2half2_rn(a, b);
  }
}

template <>
__global__ void ep_combine_kernel<__nv_bfloat16>(const __nv_bfloat16* __restrict__ y, const int32_t* __restrict__ pair_slot,
                                                 int n_tokens, int H, int W, __nv_bfloat16* __restrict__ out) {
  const long long n = static_cast<long long>(n_tokens) * (H / 2);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / (H / 2));
    const int c2 = static_cast<int>(i % (H / 2));
    float a = 0.f, b = 0.f;
    for (int r = 0; r < W; ++r) {
      const int s = pair_slot[static_cast<long long>(t) * W + r];
      if (s >= 0) {
        const float2 f = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(y + static_cast<size_t>(s) * H)[c2]);
        a += f.x;
        b += f.y;
      }
    }
    reinterpret_cast<__nv_bfloat162*>(out + static_cast<size_t>(t) * H)[c2] = __floats2bfloat162_rn(a, b);
  }
}

}  // namespace moe
