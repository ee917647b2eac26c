// router_topk.cuh — softmax top-k routing of router logits, fused ahead of the routing alignment.
//
// The caller of the MoE path turns router logits [T, E] into top-k expert ids and weights:
// probs = softmax(logits); (vals, ids) = topk(probs, k); weights = vals / sum(vals) when
// renormalising (the routing the synthetic workloads use, softmax -> top-k -> renormalise).
// Softmax is monotone, so the top-k of the probabilities is the top-k of the logits, and with
// renormalisation the full-softmax denominator cancels: weight_j = exp(l_j - m) / sum over the
// k selected of exp(l_i - m), m the largest logit. Without renormalisation the denominator is the
// sum over all E.
//
// Selection order is total and deterministic: logits compare through an order-preserving
// integer image of their fp32 value (every bit pattern, NaN included, has a place; +0 ranks above
// -0), equal images rank the lower expert index first, and the k ids of a token come out in
// descending order. The ids are therefore bit-exact against any restatement of that order.
//
// One warp per token: lane l holds logits l, l + 32, ... in registers; each of the k rounds is a
// per-lane maximum over the untaken entries and a 5-step butterfly over 64-bit (image, index)
// keys. With `counts` the kernel also builds the alignment's per-chunk expert histogram
// (counts[e * n_chunks + r / chunk], zeroed by the caller; integer atomics, so the result does not
// depend on their order), which replaces the alignment's count pass.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace moe {

constexpr int kRouterMaxTopk = 32;
constexpr int kRouterWarps = 8;

__device__ __forceinline__ uint32_t router_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float router_unkey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
__device__ __forceinline__ float router_load(const float* p) { return __ldg(p); }
__device__ __forceinline__ float router_load(const __half* p) { return __half2float(__ldg(p)); }
__device__ __forceinline__ float router_load(const __nv_bfloat16* p) { return __bfloat162float(__ldg(p)); }

__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// VPL = logits per lane (E <= 32 * VPL); topk <= min(E, kRouterMaxTopk).
template <typename LogitT, int VPL>
__global__ void __launch_bounds__(kRouterWarps * 32)
    router_topk_kernel(const LogitT* __restrict__ logits, int T, int E, int topk, int renormalize,
                       int32_t* __restrict__ ids, float* __restrict__ weights, int* __restrict__ counts, int chunk,
                       int n_chunks) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long t = warp_id; t < T; t += n_warps) {
    const LogitT* row = logits + t * E;
    uint32_t key[VPL];
    uint32_t taken = 0;  // bit i: entry lane + 32 i is selected already or does not exist
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E) {
        key[i] = router_key(router_load(row + e));
      } else {
        key[i] = 0u;
        taken |= 1u << i;
      }
    }
    const uint32_t absent = taken;
    int my_e = 0;
    float my_v = 0.f, m = 0.f;
    for (int j = 0; j < topk; ++j) {
      // key of an entry: image in the high word, 0xffffffff - index in the low word, so the
      // maximum is the largest logit and, among equal ones, the lowest index; every existing
      // entry's key is > 0, so a lane with nothing left (0) never wins
      unsigned long long best = 0ull;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const unsigned long long c =
            (static_cast<unsigned long long>(key[i]) << 32) | (0xffffffffu - static_cast<uint32_t>(lane + 32 * i));
        if (!((taken >> i) & 1u) && c > best) best = c;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      const int e = static_cast<int>(0xffffffffu - static_cast<uint32_t>(best & 0xffffffffull));
      const float v = router_unkey(static_cast<uint32_t>(best >> 32));
      if (j == 0) m = v;
      if ((e & 31) == lane) taken |= 1u << (e >> 5);
      if (lane == j) {
        my_e = e;
        my_v = v;
      }
    }
    const float p = lane < topk ? expf(my_v - m) : 0.f;
    float den;
    if (renormalize) {
      den = warp_sum_f32(p);
    } else {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < VPL; ++i)
        if (!((absent >> i) & 1u)) s += expf(router_unkey(key[i]) - m);
      den = warp_sum_f32(s);
    }
    if (lane < topk) {
      const long long r = t * topk + lane;
      ids[r] = my_e;
      weights[r] = p / den;
      if (counts) atomicAdd(&counts[static_cast<long long>(my_e) * n_chunks + r / chunk], 1);
    }
  }
}

// Group-limited sigmoid routing (the DeepSeek-V3 router): s = sigmoid(logit); selection scores
// c = s + bias[e] (bias optional); each of n_group equal expert groups scores the sum of its two
// largest c; the topk_group best groups stay eligible; the topk largest c among their experts are
// chosen (descending; ties: lower id, same total order as above); weight = s of the chosen expert,
// divided by the sum of the chosen s (+1e-20) when renormalising, times `scale`.
// One warp per token; the warp's c values pass through shared memory to the lanes that score the
// groups (lane g scores group g, n_group <= 32). Dynamic shared memory: kRouterWarps * E floats.
template <typename LogitT, int VPL>
__global__ void __launch_bounds__(kRouterWarps * 32)
    router_grouped_kernel(const LogitT* __restrict__ logits, const float* __restrict__ bias, int T, int E,
                          int n_group, int topk_group, int topk, int renormalize, float scale,
                          int32_t* __restrict__ ids, float* __restrict__ weights) {
  extern __shared__ float router_c[];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  float* cs = router_c + static_cast<size_t>(wib) * E;
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const int gsz = E / n_group;
  for (long long t = warp_id; t < T; t += n_warps) {
    const LogitT* row = logits + t * E;
    float sv[VPL];
    uint32_t key[VPL];
    uint32_t taken = 0;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E) {
        sv[i] = 1.0f / (1.0f + expf(-router_load(row + e)));
        const float c = sv[i] + (bias ? __ldg(bias + e) : 0.0f);
        key[i] = router_key(c);
        cs[e] = c;
      } else {
        sv[i] = 0.0f;
        key[i] = 0u;
        taken |= 1u << i;
      }
    }
    __syncwarp();
    // group score of group `lane`: sum of its two largest c
    unsigned long long gbest = 0ull;
    if (lane < n_group) {
      float m1 = -INFINITY, m2 = -INFINITY;
      uint32_t k1 = 0u, k2 = 0u;  // keys of m1, m2 (order of fp32 values, NaN included)
      for (int j = 0; j < gsz; ++j) {
        const float c = cs[lane * gsz + j];
        const uint32_t kc = router_key(c);
        if (j == 0 || kc > k1) {
          m2 = m1;
          k2 = k1;
          m1 = c;
          k1 = kc;
        } else if (j == 1 || kc > k2) {
          m2 = c;
          k2 = kc;
        }
      }
      const float g = gsz > 1 ? m1 + m2 : m1;
      gbest = (static_cast<unsigned long long>(router_key(g)) << 32) | (0xffffffffu - static_cast<uint32_t>(lane));
    }
    __syncwarp();  // the shared c values are read before the next token overwrites them
    // the topk_group best groups (same total order as the experts)
    uint32_t groups = 0u;
    unsigned long long gk = gbest;
    for (int r = 0; r < topk_group; ++r) {
      unsigned long long b = gk;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
        b = other > b ? other : b;
      }
      const int g = static_cast<int>(0xffffffffu - static_cast<uint32_t>(b & 0xffffffffull));
      groups |= 1u << g;
      if (lane == g) gk = 0ull;
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !((groups >> (e / gsz)) & 1u)) taken |= 1u << i;
    }
    int my_e = 0;
    float my_s = 0.f;
    for (int j = 0; j < topk; ++j) {
      unsigned long long best = 0ull;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const unsigned long long c =
            (static_cast<unsigned long long>(key[i]) << 32) | (0xffffffffu - static_cast<uint32_t>(lane + 32 * i));
        if (!((taken >> i) & 1u) && c > best) best = c;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      const int e = static_cast<int>(0xffffffffu - static_cast<uint32_t>(best & 0xffffffffull));
      float mine = 0.f;
#pragma unroll
      for (int i = 0; i < VPL; ++i)
        if (i == (e >> 5)) mine = sv[i];
      const float s_e = __shfl_sync(0xffffffffu, mine, e & 31);
      if ((e & 31) == lane) taken |= 1u << (e >> 5);
      if (lane == j) {
        my_e = e;
        my_s = s_e;
      }
    }
    const float p = lane < topk ? my_s : 0.f;
    const float den = renormalize ? warp_sum_f32(p) + 1e-20f : 1.0f;
    if (lane < topk) {
      const long long r = t * topk + lane;
      ids[r] = my_e;
      weights[r] = p / den * scale;
    }
  }
}

}  // namespace moe
