// ordered_combine.cuh — the deterministic top-k combine of the fused MoE.
//
// The default fused path adds each route's down-projection row into the token's output with
// vector red.add in Stage2's epilogue: fast, but the order of the additions (and so the last bits
// of the fp16/bf16 result) depends on which CTA finishes first. The ordered combine instead runs
// Stage2 in the reference's own padded-store form (kStage2Pad: y[p] = D * routed weight for valid
// rows, the layout submission.py:317-357 writes) and then sums each token's k rows in route order
// (j = 0 .. k-1) in fp32, rounding once. Same inputs, same bits, on every run.
//
//   raw_weights_kernel      topk_weights (token-major) -> raw expert-grouped order, the order the
//                           padded-store epilogue indexes (group_offsets[e] + i)
//   combine_ordered_kernel  out[t] = sum_j y[route_slot[t * k + j]] (slot < 0: skipped)
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace moe {

// raw[go[e] + i] = topk_weights[sorted[gpo[e] + i]] for every valid padded row p = gpo[e] + i.
__global__ void raw_weights_kernel(const void* __restrict__ tw, int w_dtype, const int32_t* __restrict__ sorted,
                                   const int32_t* __restrict__ gidx, const int32_t* __restrict__ go,
                                   const int32_t* __restrict__ gpo, const int32_t* __restrict__ meta, int R,
                                   long long P_max, int block_m, float* __restrict__ raw) {
  const long long P = min(static_cast<long long>(meta[0]), P_max);
  for (long long p = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; p < P;
       p += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int route = sorted[p];
    if (route < 0 || route >= R) continue;
    const int e = gidx[p / block_m];
    const long long q = static_cast<long long>(go[e]) + (p - gpo[e]);
    if (q >= 0 && q < R) raw[q] = load_weight(tw, w_dtype, route);
  }
}

template <typename T>
__device__ __forceinline__ void acc8(float* a, uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f;
    if constexpr (Elt<T>::kBF16) {
      f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    } else {
      f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    }
    a[2 * i] += f.x;
    a[2 * i + 1] += f.y;
  }
}

// One warp per token; lanes stride over the row's 16-byte vectors.
template <typename T>
__global__ void __launch_bounds__(256)
    combine_ordered_kernel(const T* __restrict__ y, const int32_t* __restrict__ route_slot, int T_tokens, int topk,
                           int H, T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const int vecs = H / 8;
  for (long long t = warp_id; t < T_tokens; t += n_warps) {
    const int32_t* slots = route_slot + t * topk;
    uint4* dst = reinterpret_cast<uint4*>(out + t * static_cast<long long>(H));
    for (int v = lane; v < vecs; v += 32) {
      float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < topk; ++j) {
        const int s = slots[j];
        if (s < 0) continue;
        acc8<T>(a, __ldg(reinterpret_cast<const uint4*>(y + static_cast<long long>(s) * H) + v));
      }
      dst[v] = make_uint4(Elt<T>::pack2(a[0], a[1]), Elt<T>::pack2(a[2], a[3]), Elt<T>::pack2(a[4], a[5]),
                          Elt<T>::pack2(a[6], a[7]));
    }
  }
}

}  // namespace moe
