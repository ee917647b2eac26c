// route_align.cuh — routing metadata for the grouped expert GEMMs, computed on the device.
//
// Given the flat top-k expert ids of R = T*k routes, build exactly the metadata the reference
// harness builds with torch (SUB/benchmark/remote_bench.py:82-101; race_stress2.py:65-69):
//   group_sizes[e]          = number of routes to expert e
//   group_offsets           = [0, cumsum(group_sizes)]
//   group_padded_offsets    = [0, cumsum(ceil(group_sizes / block_m) * block_m)]
//   group_idx_for_bx        = repeat_interleave(arange(E), padded_sizes / block_m)
// plus the permutation the stacked layout implies:
//   sorted_route_ids[p]     = route id (t*k + j) placed in padded row p, R for padding rows;
//                             within an expert routes keep increasing route-id order, i.e. the
//                             order of a stable argsort of the flat ids
//   route_slot[r]           = padded row of route r, -1 if its id is outside [0, E)
//   meta[0] = total padded rows P, meta[1] = number of blocks P / block_m
//
// Three launches, all bit-exact (integer counting, no floating point, no order-dependent atomics
// in the placement):
//   count    one warp per chunk of routes builds a per-chunk histogram (shared-memory atomics);
//   scan     one CTA turns the (expert-major) chunk histograms into per-chunk exclusive bases,
//            one warp per expert row, then scans the expert totals and writes the offsets, the
//            block->expert map and the padding sentinels;
//   scatter  one warp per chunk walks its routes in order, 32 at a time; __match_any_sync groups
//            equal ids, the rank inside a group is the popcount of lower lanes, so every route
//            lands at base[e] + (routes to e before it).
// Ids outside [0, E) are skipped (expert-parallel ranks pass -1 for experts they do not own).
#pragma once
#include <cstdint>

namespace moe {

constexpr int kAlignWarps = 8;          // chunks (warps) per CTA
constexpr int kAlignMaxExperts = 1024;  // shared histogram capacity per warp

template <typename IdT>
__global__ void __launch_bounds__(kAlignWarps * 32)
    align_count_kernel(const IdT* __restrict__ ids, int R, int E, int chunk, int n_chunks, int* __restrict__ counts) {
  extern __shared__ int hist[];  // [kAlignWarps][E]
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kAlignWarps * E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int c = blockIdx.x * kAlignWarps + w;
  if (c < n_chunks) {
    int* h = hist + w * E;
    const int start = c * chunk;
    const int end = min(start + chunk, R);
    for (int i = start + lane; i < end; i += 32) {
      const long long id = static_cast<long long>(ids[i]);
      if (id >= 0 && id < E) atomicAdd(&h[id], 1);
    }
    __syncwarp();
    for (int e = lane; e < E; e += 32) counts[static_cast<size_t>(e) * n_chunks + c] = h[e];  // expert-major
  }
}

// One CTA of 1024 threads. counts[e][c] (expert-major) becomes the exclusive prefix over chunks:
// each warp scans one expert's chunk row at a time, each lane a contiguous segment of it.
__global__ void __launch_bounds__(1024)
    align_scan_kernel(int* __restrict__ counts, int n_chunks, int E, int block_m, int R, int32_t* __restrict__ group_sizes,
                      int32_t* __restrict__ group_offsets, int32_t* __restrict__ group_padded_offsets,
                      int32_t* __restrict__ group_idx_for_bx, int32_t* __restrict__ sorted_route_ids,
                      int32_t* __restrict__ meta) {
  __shared__ int s_tot[kAlignMaxExperts];
  __shared__ int s_pad[kAlignMaxExperts];
  __shared__ int s_wsum[2][32];
  const int tid = threadIdx.x;
  const int lane = tid & 31, w = tid >> 5;
  // 1. per-expert totals and per-chunk exclusive bases
  const int seg = (n_chunks + 31) / 32;
  for (int e = w; e < E; e += 32) {
    int* row = counts + static_cast<size_t>(e) * n_chunks;
    const int c0 = min(lane * seg, n_chunks), c1 = min(c0 + seg, n_chunks);
    int sum = 0;
    for (int c = c0; c < c1; ++c) sum += row[c];
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - sum;
    for (int c = c0; c < c1; ++c) {
      const int v = row[c];
      row[c] = run;
      run += v;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    if (lane == 0) {
      s_tot[e] = total;
      s_pad[e] = (total + block_m - 1) / block_m * block_m;
    }
  }
  __syncthreads();
  // 2. exclusive scans of totals and padded totals over E <= 1024 (one element per thread)
  const int tot = tid < E ? s_tot[tid] : 0;
  const int pad = tid < E ? s_pad[tid] : 0;
  int it = tot, ip = pad;  // inclusive warp scans
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, it, o);
    const int b = __shfl_up_sync(0xffffffffu, ip, o);
    if (lane >= o) {
      it += a;
      ip += b;
    }
  }
  if (lane == 31) {
    s_wsum[0][w] = it;
    s_wsum[1][w] = ip;
  }
  __syncthreads();
  if (w == 0) {
    int a = s_wsum[0][lane], b = s_wsum[1][lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, a, o);
      const int y = __shfl_up_sync(0xffffffffu, b, o);
      if (lane >= o) {
        a += x;
        b += y;
      }
    }
    s_wsum[0][lane] = a;  // inclusive over warps
    s_wsum[1][lane] = b;
  }
  __syncthreads();
  const int excl_t = it - tot + (w > 0 ? s_wsum[0][w - 1] : 0);
  const int excl_p = ip - pad + (w > 0 ? s_wsum[1][w - 1] : 0);
  const int total_valid = s_wsum[0][31];
  const int total_padded = s_wsum[1][31];
  if (tid < E) {
    group_sizes[tid] = tot;
    group_offsets[tid] = excl_t;
    group_padded_offsets[tid] = excl_p;
    // block -> expert map and padding sentinels of this expert
    if (group_idx_for_bx) {
      for (int b = excl_p / block_m; b < (excl_p + pad) / block_m; ++b) group_idx_for_bx[b] = tid;
    }
    for (int s = excl_p + tot; s < excl_p + pad; ++s) sorted_route_ids[s] = R;
  }
  if (tid == 0) {
    group_offsets[E] = total_valid;
    group_padded_offsets[E] = total_padded;
    meta[0] = total_padded;
    meta[1] = total_padded / block_m;
    meta[2] = total_valid;
    meta[3] = 0;
  }
}

template <typename IdT>
__global__ void __launch_bounds__(kAlignWarps * 32)
    align_scatter_kernel(const IdT* __restrict__ ids, int R, int E, int chunk, int n_chunks,
                         const int* __restrict__ counts, const int32_t* __restrict__ group_padded_offsets,
                         int32_t* __restrict__ sorted_route_ids, int32_t* __restrict__ route_slot) {
  extern __shared__ int base[];  // [kAlignWarps][E]
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * kAlignWarps + w;
  if (c >= n_chunks) return;
  int* b = base + w * E;
  for (int e = lane; e < E; e += 32) b[e] = counts[static_cast<size_t>(e) * n_chunks + c] + group_padded_offsets[e];
  __syncwarp();
  const unsigned lt_mask = (1u << lane) - 1u;
  const int start = c * chunk;
  const int end = min(start + chunk, R);
  for (int s0 = start; s0 < end; s0 += 32) {
    const int r = s0 + lane;
    long long id = -1;
    if (r < end) id = static_cast<long long>(ids[r]);
    const bool valid = r < end && id >= 0 && id < E;
    const int key = valid ? static_cast<int>(id) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    int slot = -1;
    if (valid) {
      slot = b[key] + __popc(peers & lt_mask);
      sorted_route_ids[slot] = r;
    }
    if (r < end) route_slot[r] = slot;
    __syncwarp();
    if (valid && lane == 31 - __clz(peers)) b[key] += __popc(peers);
    __syncwarp();
  }
}

}  // namespace moe
