// ep_p2p.cuh — expert parallelism over peer memory: one process per GPU, every rank's "region"
// mapped into every other rank by CUDA IPC, NVLink loads for the data path and one bounded
// flag barrier on each side of the local MoE. No collectives library and no host
// synchronisation in a forward.
//
// Region of rank s (layout in EpRegion, identical on every rank):
//   sig[W]            barrier epochs written by the peers (slot q written by rank q)
//   tcount            this forward's token count of rank s
//   x[T_max, H]       rank s's hidden states
//   ids[T_max, k]     rank s's top-k expert ids (int32)
//   w[T_max, k]       rank s's top-k weights (fp32)
//   y[max(W, k) * T_max, H]
//                     pull combine: partial outputs rank s computed for every rank's tokens, row
//                     q * T_max + t = sum over rank s's experts among token (q, t)'s top-k of
//                     weight * expert(x); push combine: row t * k + j = slot j of rank s's own
//                     token t, stored by the rank that owns that expert
// A forward on rank s: stage its inputs in its region -> barrier -> route every rank's (token,
// slot) pairs whose expert it owns onto its local experts (reading the peers' ids and weights),
// gather those token rows from the peers' x, run the grouped GEMMs, Stage2 combining into its own
// y -> barrier -> out[t] = sum over the owners o of token t's experts of y_o[s * T_max + t], read
// from the owners' regions in ascending rank order (deterministic given the partials).
// Peer data is read with L2-only loads (ld.global.cg); in this (pull) mode nothing but the barrier
// flags is written to peer memory, and no load uses a tensor map or cluster multicast.
//
// Push combine (moe_ep_p2p_compute_push): Stage2's epilogue on every owner stores each route's
// weighted row straight into its slot t * k + j of the home rank's y (16-byte stores to peer
// memory, tile by tile, overlapping the GEMM; no atomics: every slot has exactly one writer);
// each epilogue thread fences at system scope before its kernel ends; after the second barrier the
// home rank sums its token's slots locally, in slot order, in fp32 (ep_push_combine_kernel,
// moe_ep_p2p_push_finish). The pull kernel and its NVLink reads after the second barrier
// disappear; the routes' rows cross NVLink during the GEMM instead.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace moe {

struct EpRegion {
  long long sig, tcount, x, ids, w, y, total;  // byte offsets
};

__host__ __device__ inline long long ep_round256(long long v) { return (v + 255) / 256 * 256; }

__host__ __device__ inline EpRegion ep_region_layout(long long T_max, long long H, long long topk, long long W) {
  EpRegion L{};
  L.sig = 0;
  L.tcount = ep_round256(W * 4);
  L.x = 1024 > L.tcount + 256 ? 1024 : ep_round256(L.tcount + 4);
  L.ids = ep_round256(L.x + T_max * H * 2);
  L.w = ep_round256(L.ids + T_max * topk * 4);
  L.y = ep_round256(L.w + T_max * topk * 4);
  L.total = ep_round256(L.y + (W > topk ? W : topk) * T_max * H * 2);
  return L;
}

template <typename T>
__device__ __forceinline__ const T* ep_at(const uint64_t* regions, int rank, long long off) {
  return reinterpret_cast<const T*>(regions[rank] + static_cast<uint64_t>(off));
}

// Copy this rank's inputs into its region: x rows (16-byte vectors), ids as int32, weights as
// fp32, and the token count.
template <typename T, typename IdT>
__global__ void ep_stage_kernel(uint8_t* __restrict__ region, EpRegion L, const T* __restrict__ x,
                                const IdT* __restrict__ ids, const void* __restrict__ w, int w_dtype, int tokens, int H,
                                int topk) {
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long nth = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long nvec = static_cast<long long>(tokens) * H / 8;
  const uint4* src = reinterpret_cast<const uint4*>(x);
  uint4* dst = reinterpret_cast<uint4*>(region + L.x);
  for (long long i = tid; i < nvec; i += nth) dst[i] = src[i];
  int32_t* rid = reinterpret_cast<int32_t*>(region + L.ids);
  float* rw = reinterpret_cast<float*>(region + L.w);
  const long long nk = static_cast<long long>(tokens) * topk;
  for (long long i = tid; i < nk; i += nth) {
    const long long e = static_cast<long long>(ids[i]);
    rid[i] = (e >= 0 && e < 0x7fffffff) ? static_cast<int32_t>(e) : -1;
    float v;
    if (w_dtype == 0)
      v = reinterpret_cast<const float*>(w)[i];
    else if (w_dtype == 1)
      v = __half2float(reinterpret_cast<const __half*>(w)[i]);
    else
      v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[i]);
    rw[i] = v;
  }
  if (tid == 0) *reinterpret_cast<int32_t*>(region + L.tcount) = tokens;
}

// Barrier over the W ranks: thread q < W stores `epoch` into rank q's slot for this rank
// (release, system scope), then waits until rank q has stored `epoch` (or later) into this
// rank's slot q (acquire, system scope). Bounded: after kEpBarrierWaitNs the wait gives up and
// flags the status word. The bound is far above the pipeline waits' because the ranks' host
// threads enqueue their forwards independently (pinning host memory or other host work can put
// one rank seconds behind another). Launched as one block of 32 threads per rank, each on its
// own GPU.
constexpr uint64_t kEpBarrierWaitNs = 60ull * 1000000000ull;

__global__ void ep_barrier_kernel(const uint64_t* __restrict__ regions, long long sig_off, int rank, int W,
                                  uint32_t epoch, uint32_t* status) {
  const int q = threadIdx.x;
  if (q < W) {
    uint32_t* slot = reinterpret_cast<uint32_t*>(regions[q] + static_cast<uint64_t>(sig_off)) + rank;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(slot), "r"(epoch) : "memory");
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(regions[rank] + static_cast<uint64_t>(sig_off)) + q;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if (static_cast<int32_t>(v - epoch) >= 0) break;
      if (globaltimer_ns() - t0 > kEpBarrierWaitNs) {
        if (status) atomicOr(status, kStatusWaitTimeout);
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// Virtual route r = (s * T_max + t) * k + j covers slot j of token t of rank s. local_ids[r] =
// this rank's local index of that expert if this rank owns it (and t < rank s's token count),
// else -1; local_w[r] = its routing weight.
__global__ void ep_p2p_route_kernel(const uint64_t* __restrict__ regions, EpRegion L, int W, int T_max, int topk,
                                    const int32_t* __restrict__ expert_rank, const int32_t* __restrict__ expert_local,
                                    int E, int rank, int32_t* __restrict__ local_ids, float* __restrict__ local_w) {
  const long long per_rank = static_cast<long long>(T_max) * topk;
  const long long n = per_rank * W;
  for (long long r = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; r < n;
       r += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(r / per_rank);
    const long long i = r - s * per_rank;  // t * k + j inside rank s
    const int tokens = __ldcg(ep_at<int32_t>(regions, s, L.tcount));
    int lid = -1;
    float wv = 0.0f;
    if (i / topk < tokens) {
      const int e = __ldcg(ep_at<int32_t>(regions, s, L.ids) + i);
      if (e >= 0 && e < E && expert_rank[e] == rank) {
        lid = expert_local[e];
        wv = __ldcg(ep_at<float>(regions, s, L.w) + i);
      }
    }
    local_ids[r] = lid;
    local_w[r] = wv;
  }
}

// xs[route_slot[r]] = x row of token (s, t) of route r, read from rank s's region; and, with
// zero_served (pull combine), zero this rank's y rows of every token with at least one local route
// (the Stage2 combine target). One warp per work item, 16-byte vectors.
template <typename T>
__global__ void gather_rows_peer_kernel(const uint64_t* __restrict__ regions, EpRegion L, int rank, int T_max,
                                        int topk, int W, const int32_t* __restrict__ route_slot,
                                        const int32_t* __restrict__ local_ids, int H, T* __restrict__ xs,
                                        int zero_served) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const int vecs = H / 8;
  const long long R = static_cast<long long>(W) * T_max * topk;
  const long long rows = zero_served ? static_cast<long long>(W) * T_max : 0;
  uint4* y = reinterpret_cast<uint4*>(regions[rank] + static_cast<uint64_t>(L.y));
  for (long long item = warp_id; item < R + rows; item += n_warps) {
    if (item < R) {
      const int slot = route_slot[item];
      if (slot < 0) continue;
      const long long tok = item / topk;  // s * T_max + t
      const int s = static_cast<int>(tok / T_max);
      const long long t = tok - static_cast<long long>(s) * T_max;
      const uint4* src = ep_at<uint4>(regions, s, L.x) + t * vecs;
      uint4* dst = reinterpret_cast<uint4*>(xs + static_cast<size_t>(slot) * H);
      // eight 16-byte loads in flight per lane: peer reads cross NVLink with microseconds of latency
      constexpr int U = 8;
      for (int v0 = lane; v0 < vecs; v0 += 32 * U) {
        uint4 tmp[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (v0 + u * 32 < vecs) tmp[u] = __ldcg(src + v0 + u * 32);
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (v0 + u * 32 < vecs) dst[v0 + u * 32] = tmp[u];
      }
    } else {
      const long long tok = item - R;
      bool served = false;
      for (int j = 0; j < topk; ++j) served |= local_ids[tok * topk + j] >= 0;
      if (!served) continue;
      uint4* dst = y + tok * vecs;
      for (int v = lane; v < vecs; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
    }
  }
}

// Deduplicating variant of gather_rows_peer_kernel (selected with MOE_B200_EP_GATHER=dedup,
// topk <= 32): one warp per virtual token (s, t) instead of per route. A token usually has several
// of its top-k experts on one rank (top-8 over 2 ranks: ~4), and the per-route kernel reads its row
// over NVLink once per route; here the warp reads it once and stores it into every local slot of
// the token (lane j holds slot j; the slots are broadcast one by one). With zero_served it also
// zeroes the token's partial row, as gather_rows_peer_kernel does.
template <typename T>
__global__ void gather_rows_peer_dedup_kernel(const uint64_t* __restrict__ regions, EpRegion L, int rank, int T_max,
                                              int topk, int W, const int32_t* __restrict__ route_slot, int H,
                                              T* __restrict__ xs, int zero_served) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const int vecs = H / 8;
  const long long rows = static_cast<long long>(W) * T_max;
  uint4* y = reinterpret_cast<uint4*>(regions[rank] + static_cast<uint64_t>(L.y));
  for (long long tok = warp_id; tok < rows; tok += n_warps) {
    const int my_slot = lane < topk ? route_slot[tok * topk + lane] : -1;
    const unsigned local = __ballot_sync(0xffffffffu, my_slot >= 0);
    if (local == 0u) continue;
    const int s = static_cast<int>(tok / T_max);
    const long long t = tok - static_cast<long long>(s) * T_max;
    const uint4* src = ep_at<uint4>(regions, s, L.x) + t * vecs;
    constexpr int U = 8;  // 16-byte loads in flight per lane
    for (int v0 = lane; v0 < vecs; v0 += 32 * U) {
      uint4 tmp[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (v0 + u * 32 < vecs) tmp[u] = __ldcg(src + v0 + u * 32);
      for (unsigned m = local; m != 0u; m &= m - 1u) {
        const int j = __ffs(static_cast<int>(m)) - 1;
        const int slot = __shfl_sync(0xffffffffu, my_slot, j);
        uint4* dst = reinterpret_cast<uint4*>(xs + static_cast<size_t>(slot) * H);
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (v0 + u * 32 < vecs) dst[v0 + u * 32] = tmp[u];
      }
    }
    if (zero_served) {
      uint4* dst = y + tok * vecs;
      for (int v = lane; v < vecs; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
    }
  }
}

// Bulk-copy variant of gather_rows_peer_kernel (selected with MOE_B200_EP_GATHER=bulk): lane 0
// of each warp moves whole token rows with the bulk-copy engine, peer row -> shared memory
// (cp.async.bulk with an mbarrier) -> xs (cp.async.bulk store), two rows in flight per warp. Then
// all threads zero the served partial rows as in gather_rows_peer_kernel (with zero_served). Dynamic
// shared memory:
// kEpBulkWarps * 2 rows of H * 2 bytes, plus the mbarriers.
constexpr int kEpBulkWarps = 4;
__device__ __forceinline__ void bulk_load_row(uint32_t dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst_smem),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_store_row(void* dst, uint32_t src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src_smem), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_reads() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <typename T>
__global__ void __launch_bounds__(kEpBulkWarps * 32)
    gather_rows_peer_bulk_kernel(const uint64_t* __restrict__ regions, EpRegion L, int rank, int T_max, int topk,
                                 int W, const int32_t* __restrict__ route_slot, const int32_t* __restrict__ local_ids,
                                 int H, T* __restrict__ xs, uint32_t* status, int zero_served) {
  extern __shared__ __align__(128) uint8_t ep_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t row_bytes = static_cast<uint32_t>(H) * 2u;
  uint8_t* buf = ep_smem + static_cast<size_t>(warp) * 2 * row_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ep_smem + static_cast<size_t>(kEpBulkWarps) * 2 * row_bytes) + 2 * warp;
  const long long R = static_cast<long long>(W) * T_max * topk;
  const long long gw = static_cast<long long>(blockIdx.x) * kEpBulkWarps + warp;
  const long long nw = static_cast<long long>(gridDim.x) * kEpBulkWarps;
  if (lane == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
    auto next_valid = [&](long long r) {
      while (r < R && route_slot[r] < 0) r += nw;
      return r;
    };
    auto src_of = [&](long long r) {
      const long long tok = r / topk;  // s * T_max + t
      const int s = static_cast<int>(tok / T_max);
      const long long t = tok - static_cast<long long>(s) * T_max;
      return reinterpret_cast<const uint8_t*>(regions[s] + static_cast<uint64_t>(L.x)) + t * row_bytes;
    };
    uint32_t phase[2] = {0u, 0u};
    bool pending[2] = {false, false};  // a load into the buffer has been issued and not yet seen to land
    long long cur = next_valid(gw);
    int sb = 0;
    if (cur < R) {
      mbar_arrive_expect_tx(&bars[0], row_bytes);
      bulk_load_row(smem_u32(buf), src_of(cur), row_bytes, &bars[0]);
      pending[0] = true;
    }
    bool ok = true;
    while (cur < R && ok) {
      const long long nxt = next_valid(cur + nw);
      const int nb = sb ^ 1;
      if (nxt < R) {
        bulk_wait_reads();  // the store that last used buffer nb has read it
        mbar_arrive_expect_tx(&bars[nb], row_bytes);
        bulk_load_row(smem_u32(buf + nb * row_bytes), src_of(nxt), row_bytes, &bars[nb]);
        pending[nb] = true;
      }
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&bars[sb], phase[sb])) {
        if (globaltimer_ns() - t0 > MOE_WAIT_NS) {
          if (status) atomicOr(status, kStatusWaitTimeout);
          ok = false;
          break;
        }
      }
      if (!ok) break;
      phase[sb] ^= 1u;
      pending[sb] = false;
      const int slot = route_slot[cur];
      bulk_store_row(xs + static_cast<size_t>(slot) * H, smem_u32(buf + sb * row_bytes), row_bytes);
      cur = nxt;
      sb = nb;
    }
    // after a timeout, wait (bounded) only for the loads still outstanding, then for every store;
    // a load that has not landed by then leaves xs undefined, which the status word reports
    for (int b = 0; b < 2; ++b) {
      const uint64_t t0 = globaltimer_ns();
      while (pending[b] && !mbar_try_wait(&bars[b], phase[b]) && globaltimer_ns() - t0 < MOE_WAIT_NS) {
      }
    }
    bulk_wait_all();
  }
  __syncwarp();
  // zero this rank's partial rows of every token with at least one local route
  const int vecs = H / 8;
  const long long rows = zero_served ? static_cast<long long>(W) * T_max : 0;
  uint4* y = reinterpret_cast<uint4*>(regions[rank] + static_cast<uint64_t>(L.y));
  for (long long tok = gw; tok < rows; tok += nw) {
    bool served = false;
    for (int j = 0; j < topk; ++j) served |= local_ids[tok * topk + j] >= 0;
    if (!served) continue;
    uint4* dst = y + tok * vecs;
    for (int v = lane; v < vecs; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
  }
}

// Push combine, home side: out[t] = sum over token t's slots j whose expert id is in [0, E) (each
// written by that expert's owner) of y[t * k + j], in slot order, accumulated in fp32. One warp
// per token, 8 elements per lane step; all of a token's slots are loaded before the sum.
template <typename T>
__global__ void ep_push_combine_kernel(const uint8_t* __restrict__ region, EpRegion L, int tokens, int H, int topk,
                                       int E, T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const int vecs = H / 8;
  const int32_t* ids = reinterpret_cast<const int32_t*>(region + L.ids);
  const uint4* y = reinterpret_cast<const uint4*>(region + L.y);
  for (long long t = warp_id; t < tokens; t += n_warps) {
    const int my_e = lane < topk ? ids[t * topk + lane] : -1;
    const unsigned valid = __ballot_sync(0xffffffffu, my_e >= 0 && my_e < E);
    for (int v = lane; v < vecs; v += 32) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (unsigned m0 = valid; m0 != 0u;) {
        uint4 p[8];
        int n = 0;
        unsigned m = m0;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (m == 0u) break;
          const int j = __ffs(static_cast<int>(m)) - 1;
          m &= m - 1u;
          p[u] = y[(t * topk + j) * vecs + v];
          ++n;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (u >= n) break;
          const T* pe = reinterpret_cast<const T*>(&p[u]);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] += static_cast<float>(pe[i]);
        }
        m0 = m;
      }
      uint4 r;
      T* re = reinterpret_cast<T*>(&r);
#pragma unroll
      for (int i = 0; i < 8; ++i) re[i] = static_cast<T>(acc[i]);
      reinterpret_cast<uint4*>(out + t * static_cast<long long>(H))[v] = r;
    }
  }
}

// out[t] = sum over the distinct owner ranks o of token t's experts (ascending o) of rank o's
// y[rank * T_max + t], accumulated in fp32. One warp per token, 8 elements per lane step.
template <typename T>
__global__ void ep_combine_pull_kernel(const uint64_t* __restrict__ regions, EpRegion L, int rank, int W, int T_max,
                                       int tokens, int H, int topk, const int32_t* __restrict__ expert_rank, int E,
                                       T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const int vecs = H / 8;
  const int32_t* ids = ep_at<int32_t>(regions, rank, L.ids);
  for (long long t = warp_id; t < tokens; t += n_warps) {
    uint32_t owners = 0;  // bit o: rank o owns one of the token's experts (W <= 32)
    for (int j = 0; j < topk; ++j) {
      const int e = ids[t * topk + j];
      if (e >= 0 && e < E) {
        const int o = expert_rank[e];
        if (o >= 0 && o < W) owners |= 1u << o;
      }
    }
    int ow[32];  // owner ranks in ascending order
    int n_ow = 0;
    for (int o = 0; o < W; ++o)
      if (owners >> o & 1u) ow[n_ow++] = o;
    const long long row = (static_cast<long long>(rank) * T_max + t) * vecs;
    for (int v = lane; v < vecs; v += 32) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      // all owners' vectors requested before any is summed (up to 8 NVLink loads in flight)
      for (int o0 = 0; o0 < n_ow; o0 += 8) {
        uint4 p[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (o0 + u < n_ow) p[u] = __ldcg(ep_at<uint4>(regions, ow[o0 + u], L.y) + row + v);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (o0 + u >= n_ow) break;
          const T* pe = reinterpret_cast<const T*>(&p[u]);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] += static_cast<float>(pe[i]);
        }
      }
      uint4 r;
      T* re = reinterpret_cast<T*>(&r);
#pragma unroll
      for (int i = 0; i < 8; ++i) re[i] = static_cast<T>(acc[i]);
      reinterpret_cast<uint4*>(out + t * static_cast<long long>(H))[v] = r;
    }
  }
}

}  // namespace moe
