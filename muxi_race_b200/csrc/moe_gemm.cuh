// moe_gemm.cuh — the grouped expert GEMM of the fused MoE, as one persistent,
// warp-specialised tcgen05 kernel template for sm_100a.
//
// One CTA per SM (192 threads):
//   warp 0      TMA producer: streams A (token rows) and B (expert weight rows) k-blocks into a
//               STAGES-deep ring of 128B-swizzled shared-memory buffers;
//   warp 1      owns TMEM (512 columns = two 128x256 fp32/int32 accumulators) and one lane issues
//               tcgen05.mma for each k-block, committing to the ring's "empty" barriers;
//   warps 2..5  epilogue: tcgen05.ld the finished accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31 = tile rows), apply the fused epilogue, store to global, and hand
//               the accumulator back, so the epilogue of tile i overlaps the main loop of tile i+1.
//
// Tiles are 128 rows (one routing block = one expert) x 256 accumulator columns, k-blocks are
// 128 bytes wide (64 fp16/bf16 or 128 int8 elements), four MMAs of K = 128 bytes / 4 each.
// Tile t covers routing block t / n_tiles and column tile t % n_tiles: all column tiles of a block
// run back to back (the A block is re-read from L2) and the blocks of one expert are adjacent
// (its weight tile is re-read from L2, not HBM).
//
// Modes (the epilogue is the only difference):
//   kStage1     D = [gate | up] halves of 128 columns each; U = silu(gate) * up, stored to the
//               [rows, I] intermediate (reference Stage1, SUB/submission.py:586-641);
//   kStage2Pad  out[p, :] = D * routed[route(p)] for valid rows and 0 for pad rows, in the
//               padded stacked layout (reference Stage2, SUB/submission.py:317-357, 933-947);
//   kStage2Comb out[token(p), :] += D * topk_weight(p) via vector red.add into the token-major
//               output (the top-k combine fused into the down GEMM's epilogue).
// Integer variants (IS_I8) dequantise the int32 accumulator with per-row (token) and per-column
// (weight output row) scales before the same epilogue.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sm100_ptx.cuh"

namespace moe {

constexpr int kBM = 128;           // rows per tile = routing block size
constexpr int kBN = 256;           // accumulator columns per tile (MMA N)
constexpr int kKBytes = 128;       // k-block width in bytes (one 128B swizzle atom)
constexpr int kStages = 4;         // smem ring depth
constexpr int kThreads = 192;      // 6 warps
constexpr int kABytes = kBM * kKBytes;        // 16 KiB
constexpr int kBBytes = kBN * kKBytes;        // 32 KiB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kTmemCols = 2 * kBN;            // double-buffered accumulator
constexpr int kSmemBytes = 1024 /*align slack*/ + kStages * kStageBytes + 256 /*barriers*/;

enum GemmMode : int { kStage1 = 0, kStage2Pad = 1, kStage2Comb = 2 };

struct GemmArgs {
  int K;                      // reduction length in elements
  int N;                      // valid output columns per expert (I for Stage1, H for Stage2)
  int n_tiles;                // column tiles per block
  int nblk;                   // routing blocks, or -1: read *nblk_dev (device-resident count)
  const int* nblk_dev;
  int E;
  const int* block_expert;    // [nblk] expert of each 128-row block (group_idx_for_bx)
  int b_rows_per_expert;      // rows of one expert in the B tensor map(s)
  int b1_row_offset;          // Stage1: row offset of the "up" half inside one expert of map B1

  // Stage1 output: U [rows, ldu]
  void* U;
  int ldu;

  // Stage2 output: out [rows or tokens, ldo]
  void* out;
  int ldo;
  // Stage2Pad: reference metadata and routed weights (fp32 or 16-bit)
  const int* group_sizes;
  const int* group_offsets;
  const int* group_padded_offsets;
  const void* routed;
  int routed_dtype;           // 0 = fp32, 1 = fp16, 2 = bf16
  int R;                      // number of routed rows (total_valid_tokens)
  // Stage2Comb: route id of each padded row (R = pad) and top-k
  const int* sorted_route_ids;
  int topk;

  // int8 dequant scales: per A row and per B output row (fp32)
  const float* a_scale;       // [rows]
  const float* b0_scale;      // [E * b_rows_per_expert] (gate rows / down rows)
  const float* b1_scale;      // [E * b_rows_per_expert] (up rows, Stage1)
  float* row_amax;            // Stage1 int8: per-row amax of U (for requantisation), may be null

  uint32_t* status;           // device status word (OR of kStatus* bits)
};

// ------------------------------------------------------------------ element helpers
template <typename T> struct Elt;
template <> struct Elt<__half> {
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static constexpr bool kBF16 = false;
};
template <> struct Elt<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static constexpr bool kBF16 = true;
};

__device__ __forceinline__ void red_add_v4(__half* p, uint4 v) {
  asm volatile("red.global.add.noftz.v4.f16x2 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void red_add_v4(__nv_bfloat16* p, uint4 v) {
  asm volatile("red.global.add.noftz.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__device__ __forceinline__ float load_weight(const void* w, int dtype, int i) {
  if (dtype == 0) return reinterpret_cast<const float*>(w)[i];
  if (dtype == 1) return __half2float(reinterpret_cast<const __half*>(w)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[i]);
}

// silu(g) * u = g / (1 + e^-g) * u; the exponential is CUDA's __expf.
__device__ __forceinline__ float silu_mul(float g, float u) { return g * __frcp_rn(1.0f + __expf(-g)) * u; }

// ------------------------------------------------------------------ the kernel
template <int MODE, typename OutT, bool IS_I8>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                    const __grid_constant__ CUtensorMap tmB1, const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + kStages * kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* full_bar = bars;                      // [kStages]
  uint64_t* empty_bar = bars + kStages;           // [kStages]
  uint64_t* tfull_bar = bars + 2 * kStages;       // [2]
  uint64_t* tempty_bar = bars + 2 * kStages + 2;  // [2]
  uint64_t* drain_bar = bars + 2 * kStages + 4;   // [1] MMA warp: all issued MMAs retired
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 4);  // one arrive per epilogue warp
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB0);
    if (MODE == kStage1) tma_prefetch_desc(&tmB1);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int nblk = args.nblk >= 0 ? args.nblk : *args.nblk_dev;
  const int num_tiles = nblk * args.n_tiles;
  const int num_kb = (args.K * (IS_I8 ? 1 : 2) + kKBytes - 1) / kKBytes;
  constexpr int kKElems = IS_I8 ? kKBytes : kKBytes / 2;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      const uint64_t pol_a = l2_policy_evict_last();    // token rows: re-read by every column tile
      const uint64_t pol_b = l2_policy_evict_normal();  // weights: re-read by the expert's other blocks
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int issued_parity[kStages];  // parity of the last load issued into each stage, -1 = none
#pragma unroll
      for (int s = 0; s < kStages; ++s) issued_parity[s] = -1;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mb = tile / args.n_tiles;
        const int nt = tile - mb * args.n_tiles;
        const int e = args.block_expert[mb];
        if (e < 0 || e >= args.E) continue;
        const int arow = mb * kBM;
        int brow0, brow1;
        if (MODE == kStage1) {
          brow0 = e * args.b_rows_per_expert + nt * (kBN / 2);
          brow1 = e * args.b_rows_per_expert + args.b1_row_offset + nt * (kBN / 2);
        } else {
          brow0 = e * args.b_rows_per_expert + nt * kBN;
          brow1 = 0;
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, args.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], kStageBytes);
          const int kx = kb * kKElems;
          tma_load_2d(smA + stage * kABytes, &tmA, &full_bar[stage], kx, arow, pol_a);
          if (MODE == kStage1) {
            tma_load_2d(smB + stage * kBBytes, &tmB0, &full_bar[stage], kx, brow0, pol_b);
            tma_load_2d(smB + stage * kBBytes + kBBytes / 2, &tmB1, &full_bar[stage], kx, brow1, pol_b);
          } else {
            tma_load_2d(smB + stage * kBBytes, &tmB0, &full_bar[stage], kx, brow0, pol_b);
          }
          issued_parity[stage] = static_cast<int>(phase);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: every load this thread issued must have landed before the CTA may exit. On the
      // normal path these phases completed long ago; after an abort this bounds the wait.
#pragma unroll
      for (int s = 0; s < kStages; ++s)
        if (issued_parity[s] >= 0) mbar_wait_drain(&full_bar[s], static_cast<uint32_t>(issued_parity[s]));
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = IS_I8 ? idesc_i8(kBM, kBN) : idesc_f16(Elt<OutT>::kBF16, kBM, kBN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mb = tile / args.n_tiles;
        const int e = args.block_expert[mb];
        if (e < 0 || e >= args.E) continue;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, args.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smA + stage * kABytes);
          const uint32_t b_addr = smem_u32(smB + stage * kBBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = smem_desc_sw128(a_addr + k * 32);
            const uint64_t bd = smem_desc_sw128(b_addr + k * 32);
            if (IS_I8)
              mma_i8(d_tmem, ad, bd, idesc, (kb | k) != 0);
            else
              mma_f16(d_tmem, ad, bd, idesc, (kb | k) != 0);
          }
          tc_commit(&empty_bar[stage]);  // frees this smem stage once the MMAs have read it
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tfull_bar[acc]);  // accumulator ready for the epilogue
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: all MMAs this thread issued retire before TMEM is released.
      tc_commit(drain_bar);
      mbar_wait_drain(drain_bar, 0);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int q = warp & 3;                  // TMEM lane quadrant this warp may access
    const int row_in_tile = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int mb = tile / args.n_tiles;
      const int nt = tile - mb * args.n_tiles;
      const int e = args.block_expert[mb];
      if (e < 0 || e >= args.E) {
        if (lane == 0 && args.status) atomicOr(args.status, kStatusBadExpert);
        continue;
      }
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, args.status)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * kBN);
      const int p = mb * kBM + row_in_tile;  // padded row of this thread

      if (MODE == kStage1) {
        OutT* U = reinterpret_cast<OutT*>(args.U);
        const int n0 = nt * (kBN / 2);
        float sa = 1.0f;
        if (IS_I8) sa = args.a_scale[p];
        float amax = 0.0f;
#pragma unroll 1
        for (int c = 0; c < kBN / 2; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(t_row + c, g);
          tmem_ld_32x32b_x32(t_row + kBN / 2 + c, u);
          tmem_ld_wait();
          const int col0 = n0 + c;
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float g0, g1, u0, u1;
            if (IS_I8) {
              const int cc = min(col0 + j, args.N - 2);
              const size_t wrow = static_cast<size_t>(e) * args.b_rows_per_expert;
              g0 = static_cast<float>(static_cast<int>(g[j])) * sa * args.b0_scale[wrow + cc];
              g1 = static_cast<float>(static_cast<int>(g[j + 1])) * sa * args.b0_scale[wrow + cc + 1];
              u0 = static_cast<float>(static_cast<int>(u[j])) * sa * args.b1_scale[wrow + args.b1_row_offset + cc];
              u1 = static_cast<float>(static_cast<int>(u[j + 1])) * sa *
                   args.b1_scale[wrow + args.b1_row_offset + cc + 1];
            } else {
              g0 = __uint_as_float(g[j]);
              g1 = __uint_as_float(g[j + 1]);
              u0 = __uint_as_float(u[j]);
              u1 = __uint_as_float(u[j + 1]);
            }
            const float h0 = silu_mul(g0, u0), h1 = silu_mul(g1, u1);
            if (IS_I8 && col0 + j < args.N) amax = fmaxf(amax, fmaxf(fabsf(h0), fabsf(h1)));
            packed[j / 2] = Elt<OutT>::pack2(h0, h1);
          }
          OutT* dst = U + static_cast<size_t>(p) * args.ldu + col0;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            if (col0 + v * 8 < args.N)
              *reinterpret_cast<uint4*>(dst + v * 8) =
                  make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
          }
        }
        if (IS_I8 && args.row_amax)
          atomicMax(reinterpret_cast<int*>(args.row_amax) + p, __float_as_int(amax));  // amax >= 0
      } else {
        // Stage2: per-row scale
        const int n0 = nt * kBN;
        float scale = 0.0f;
        bool valid = false;
        int token = 0;
        if (MODE == kStage2Pad) {
          const int local = p - args.group_padded_offsets[e];
          valid = local >= 0 && local < args.group_sizes[e];
          if (valid) {
            int route = args.group_offsets[e] + local;
            route = max(0, min(route, args.R - 1));  // reference clamp (SUB/submission.py:935-947)
            scale = load_weight(args.routed, args.routed_dtype, route);
          }
        } else {
          const int route = args.sorted_route_ids[p];
          valid = route >= 0 && route < args.R;
          if (valid) {
            token = route / args.topk;
            scale = load_weight(args.routed, args.routed_dtype, route);
          }
        }
        float sa = 1.0f;
        if (IS_I8) sa = args.a_scale[p];
        OutT* out = reinterpret_cast<OutT*>(args.out);
        const size_t orow = MODE == kStage2Pad ? static_cast<size_t>(p) : static_cast<size_t>(token);
#pragma unroll 1
        for (int c = 0; c < kBN; c += 32) {
          const int col0 = n0 + c;
          if (col0 >= args.N) break;
          uint32_t d[32];
          tmem_ld_32x32b_x32(t_row + c, d);
          tmem_ld_wait();
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float d0, d1;
            if (IS_I8) {
              const int cc = min(col0 + j, args.N - 2);
              const size_t wrow = static_cast<size_t>(e) * args.b_rows_per_expert;
              d0 = static_cast<float>(static_cast<int>(d[j])) * sa * args.b0_scale[wrow + cc];
              d1 = static_cast<float>(static_cast<int>(d[j + 1])) * sa * args.b0_scale[wrow + cc + 1];
            } else {
              d0 = __uint_as_float(d[j]);
              d1 = __uint_as_float(d[j + 1]);
            }
            packed[j / 2] = valid ? Elt<OutT>::pack2(d0 * scale, d1 * scale) : 0u;
          }
          if (MODE == kStage2Pad) {
            OutT* dst = out + orow * args.ldo + col0;
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col0 + v * 8 < args.N)
                *reinterpret_cast<uint4*>(dst + v * 8) =
                    make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
          } else if (valid) {
            OutT* dst = out + orow * args.ldo + col0;
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col0 + v * 8 < args.N)
                red_add_v4(dst + v * 8,
                           make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]));
          }
        }
      }
      // hand the accumulator back to the MMA warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace moe
