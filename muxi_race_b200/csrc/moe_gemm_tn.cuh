// moe_gemm_tn.cuh — the grouped expert GEMM with the operands swapped: the expert's weight rows
// are the MMA's M side (128 rows) and the expert's tokens its N side (a multiple of 16, at most
// 256), so a work unit pads an expert's rows only to the next multiple of 16 instead of 128.
//
// Why: with 128-row token blocks, an expert with 129..256 routed rows computes 256 rows, and on
// the DeepSeek-shaped workload (about 128 +- 11 rows per expert) a third of the tensor-core work
// is padding. Here a unit is (expert, token chunk of <= 256 rows, 128 weight rows): the weight
// tile is read once for all of the chunk's tokens and the MMA computes round16(rows) columns.
//
// Layout of one unit's accumulator (TMEM lanes = weight rows, columns = tokens):
//   Stage1  the 128 weight rows are 64 gate and 64 up rows of the same 64 features, interleaved
//           by 8-row atoms (gate 8a..8a+7, up 8a..8a+7, gate 8a+8.., ...) by one 5-D TMA box
//           {k 64, row 8, gate/up 2, row group 8, k-block 1}; TMEM lane 16a + r holds gate feature
//           8a + r and lane 16a + 8 + r its up feature, so a lane and its partner lane ^ 8 (same
//           warp) combine SiLU(gate) * up with one shuffle. Lane l of quadrant q owns feature
//           16q + 8(l >> 4) + (l & 7) and writes U[token][feature] for 32 tokens per TMEM load:
//           lanes 0 and 16 gather their eight gate lanes' results into one 16-byte store each.
//   Stage2  the 128 weight rows are 128 output features; lane m holds feature n0 + m of every
//           token: lanes 8g .. 8g+7 pack their eight features into one 16-byte reduction (combine
//           into the token-major output) or store (padded layout) issued by lane 8g.
// Roles, rings, bounded waits and drains are those of moe_gemm_kernel (warp 0 weights, warp 6
// tokens, warp 1 MMA issuer and TMEM owner, warps 2..5 epilogue); two 256-column accumulator
// slots, so an epilogue overlaps the next unit's main loop.
//
// Work units: entry = (expert, token chunk); an expert with n routed rows has ceil(n / 256)
// chunks of round16(ceil(n / chunks)) rows. Units are numbered entry-major (n_tiles weight tiles
// per entry) and, within an expert, re-ordered tile-major so that the expert's chunks read each
// weight tile at the same time.
#pragma once
#include "moe_gemm.cuh"

namespace moe {

constexpr int kTnMaxN = 256;                     // token columns per unit
constexpr int kTnWBytes = kBM * kKBytes;         // 16 KiB: 128 weight rows x one k-block
constexpr int kTnXBytes = kTnMaxN * kKBytes;     // 32 KiB: up to 256 token rows x one k-block

template <int AST, int BST> struct TnRing {
  static constexpr int kRingBytes = AST * kTnWBytes + BST * kTnXBytes;
  static_assert(kRingBytes <= kRingMax, "ring exceeds shared memory");
  static constexpr int kSmemBytes = 1024 + kRingBytes + 512;
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KiB of shared memory a CTA may opt in to");
};

struct TnArgs {
  int K;                        // reduction length (elements)
  int N;                        // valid output features per expert (I for Stage1, H for Stage2)
  int n_tiles;                  // weight tiles per expert (ceil(N / 64) Stage1, ceil(N / 128) Stage2)
  const int* n_entries_dev;     // number of (expert, chunk) entries
  const int* entries;           // [2g] expert of entry g, [2g+1] its expert's first entry
  int E;
  const int* group_sizes;       // routed rows per expert
  const int* group_offsets;     // [E+1] route offsets (Stage2Pad)
  const int* group_padded_offsets;  // [E+1] first stacked row of each expert
  int b_rows_per_expert;        // Stage2: weight rows per expert (H)
  long long w_group_per_expert; // Stage1: 8-row groups per expert in the 5-D weight map (2I / 8 or I / 8)
  void* U;                      // Stage1 output [rows, ldu]
  int ldu;
  void* out;                    // Stage2 output
  int ldo;
  const void* routed;
  int routed_dtype;             // 0 fp32, 1 fp16, 2 bf16
  int R;
  const int* sorted_route_ids;  // Stage2Comb
  int topk;
  int nblk;                     // 128-row blocks of the stacked row space
  // 8-bit kinds: per stacked row (token) and per weight row scales, Stage1 row amax of U
  const float* a_scale;         // [stacked rows]
  const float* b_scale;         // [E * b_scale_rows]
  int b_scale_rows;             // weight rows per expert in b_scale (2I Stage1, H Stage2)
  int b_up_offset;              // Stage1: the up rows' offset inside an expert (I)
  float* row_amax;              // Stage1: per stacked row amax of U (requantisation), may be null
  uint32_t* status;
};

__device__ __forceinline__ void red_add_x2(__half* p, uint32_t v) {
  asm volatile("red.global.add.noftz.f16x2 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_add_x2(__nv_bfloat16* p, uint32_t v) {
  asm volatile("red.global.add.noftz.bf16x2 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Chunking of expert e: chunks and rows per chunk (multiple of 16).
__device__ __forceinline__ void tn_chunking(int n, int& chunks, int& cs) {
  chunks = (n + kTnMaxN - 1) / kTnMaxN;
  const int per = chunks > 0 ? (n + chunks - 1) / chunks : 0;
  cs = (per + 15) / 16 * 16;
}

// Unit decode: expert, first local row and rows of the chunk, weight tile. False = skip.
__device__ __forceinline__ bool tn_unit(const TnArgs& a, int u, int& e, int& row0, int& rows, int& nt) {
  const int g0 = u / a.n_tiles;
  e = a.entries[2 * g0];
  const int gs = a.entries[2 * g0 + 1];  // the expert's first entry
  if (e < 0 || e >= a.E || gs < 0 || gs > g0) return false;
  const int n = a.group_sizes[e];
  int chunks, cs;
  tn_chunking(n, chunks, cs);
  if (chunks < 1) return false;
  const int local = u - gs * a.n_tiles;
  if (local < 0 || local >= chunks * a.n_tiles) return false;
  nt = local / chunks;
  const int c = local - nt * chunks;
  row0 = c * cs;
  rows = min(cs, n - row0);
  if (rows <= 0) return false;
  const int base = a.group_padded_offsets[e];
  return base >= 0 && base + row0 + rows <= a.nblk * kBM;
}

// The token rows [r0, r0 + N) of one k-block as boxes of 128 / 64 / 32 / 16 rows.
__device__ __forceinline__ void tn_load_x(uint8_t* dst, const CUtensorMap* m128, const CUtensorMap* m64,
                                          const CUtensorMap* m32, const CUtensorMap* m16, uint64_t* bar, int kx, int r0,
                                          int N, uint64_t pol) {
  int off = 0;
  while (N - off >= 128) {
    tma_load_2d(dst + off * kKBytes, m128, bar, kx, r0 + off, pol);
    off += 128;
  }
  if (N - off >= 64) {
    tma_load_2d(dst + off * kKBytes, m64, bar, kx, r0 + off, pol);
    off += 64;
  }
  if (N - off >= 32) {
    tma_load_2d(dst + off * kKBytes, m32, bar, kx, r0 + off, pol);
    off += 32;
  }
  if (N - off >= 16) tma_load_2d(dst + off * kKBytes, m16, bar, kx, r0 + off, pol);
}

// tmW: Stage1 5-D map {64, 8, 2, groups, k-blocks} over the gate/up rows (box {64, 8, 2, 8, 1}),
//      Stage2 2-D map {K, rows} (box 128 rows). tmX*: the stacked token rows (Stage1 xs, Stage2
//      U) with boxes of 128 / 64 / 32 / 16 rows.
// Q8: operand kind (kQ16, kQI8, kQF8; the 8-bit kinds dequantise with a_scale x b_scale).
template <int MODE, typename OutT, int AST, int BST, int Q8 = kQ16>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_tn_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX128,
                       const __grid_constant__ CUtensorMap tmX64, const __grid_constant__ CUtensorMap tmX32,
                       const __grid_constant__ CUtensorMap tmX16, const TnArgs args) {
  using RingT = TnRing<AST, BST>;
  constexpr int kSlots = kTmemCols / kTnMaxN;  // 2
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring_w = smem;                          // [AST][16 KiB]
  uint8_t* ring_x = smem + AST * kTnWBytes;        // [BST][32 KiB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + RingT::kRingBytes);
  uint64_t* fullW = bars;
  uint64_t* emptyW = fullW + AST;
  uint64_t* fullX = emptyW + AST;
  uint64_t* emptyX = fullX + BST;
  uint64_t* tfull_bar = emptyX + BST;
  uint64_t* tempty_bar = tfull_bar + kSlots;
  uint64_t* drain_bar = tempty_bar + kSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < AST; ++s) {
      mbar_init(&fullW[s], 1);
      mbar_init(&emptyW[s], 1);
    }
    for (int s = 0; s < BST; ++s) {
      mbar_init(&fullX[s], 1);
      mbar_init(&emptyX[s], 1);
    }
    for (int a = 0; a < kSlots; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX128);
    tma_prefetch_desc(&tmX64);
    tma_prefetch_desc(&tmX32);
    tma_prefetch_desc(&tmX16);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_units = *args.n_entries_dev * args.n_tiles;
  constexpr int kElt = Q8 ? 1 : 2;
  const int num_kb = (args.K * kElt + kKBytes - 1) / kKBytes;
  constexpr int kKElems = kKBytes / kElt;

  if (warp == 0 || warp == 6) {
    // ---------------------------------------------------------------- producers
    if (lane == 0) {
      const bool is_w = warp == 0;
      const int depth = is_w ? AST : BST;
      uint64_t* full = is_w ? fullW : fullX;
      uint64_t* empty = is_w ? emptyW : emptyX;
      const uint64_t pol = is_w ? l2_policy_evict_normal() : l2_policy_evict_last();
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      int par[AST > BST ? AST : BST];
#pragma unroll
      for (int s = 0; s < (AST > BST ? AST : BST); ++s) par[s] = -1;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int e, row0, rows, nt;
        if (!tn_unit(args, u, e, row0, rows, nt)) continue;
        const int N = (rows + 15) / 16 * 16;
        const int xrow = args.group_padded_offsets[e] + row0;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[st], ph ^ 1u, abort_flag, args.status)) {
            ok = false;
            break;
          }
          if (is_w) {
            mbar_arrive_expect_tx(&full[st], kTnWBytes);
            uint8_t* dst = ring_w + st * kTnWBytes;
            if (MODE == kStage1) {
              const int g = static_cast<int>(static_cast<long long>(e) * args.w_group_per_expert) + nt * 8;
              asm volatile(
                  "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
                  " [%0], [%1, {%3, %4, %5, %6, %7}], [%2], %8;" ::"r"(smem_u32(dst)),
                  "l"(&tmW), "r"(smem_u32(&full[st])), "r"(0), "r"(0), "r"(0), "r"(g), "r"(kb), "l"(pol)
                  : "memory");
            } else {
              tma_load_2d(dst, &tmW, &full[st], kb * kKElems, e * args.b_rows_per_expert + nt * kBM, pol);
            }
          } else {
            mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(N * kKBytes));
            tn_load_x(ring_x + st * kTnXBytes, &tmX128, &tmX64, &tmX32, &tmX16, &full[st], kb * kKElems, xrow, N,
                      pol);
          }
          par[st] = static_cast<int>(ph);
          if (++st == depth) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      for (int s = 0; s < depth; ++s)
        if (par[s] >= 0) mbar_wait_drain(&full[s], static_cast<uint32_t>(par[s]));
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc0 = (Q8 == kQF8 ? idesc_f8(kBM, 16)
                               : Q8     ? idesc_i8(kBM, 16)
                                        : idesc_f16(Elt<OutT>::kBF16, kBM, 16)) &
                              ~(0x3Fu << 17);  // N set per unit
      int sw = 0, sx = 0;
      uint32_t pw = 0, px = 0;
      uint32_t slot_cnt = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int e, row0, rows, nt;
        if (!tn_unit(args, u, e, row0, rows, nt)) continue;
        const int N = (rows + 15) / 16 * 16;
        const uint32_t idesc = idesc0 | (static_cast<uint32_t>(N >> 3) << 17);
        const int slot = static_cast<int>(slot_cnt % kSlots);
        const uint32_t use = slot_cnt / kSlots;
        ++slot_cnt;
        if (!mbar_wait(&tempty_bar[slot], (use & 1u) ^ 1u, abort_flag, args.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * kTnMaxN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&fullW[sw], pw, abort_flag, args.status) ||
              !mbar_wait(&fullX[sx], px, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t w_addr = smem_u32(ring_w + sw * kTnWBytes);
          const uint32_t x_addr = smem_u32(ring_x + sx * kTnXBytes);
#pragma unroll
          for (int k = 0; k < kKBytes / 32; ++k) {
            const uint64_t wd = smem_desc_sw128(w_addr + k * 32), xd = smem_desc_sw128(x_addr + k * 32);
            if (Q8 == kQF8)
              mma_f8(d_tmem, wd, xd, idesc, (kb | k) != 0);
            else if (Q8)
              mma_i8(d_tmem, wd, xd, idesc, (kb | k) != 0);
            else
              mma_f16(d_tmem, wd, xd, idesc, (kb | k) != 0);
          }
          tc_commit(&emptyW[sw]);
          tc_commit(&emptyX[sx]);
          if (++sw == AST) {
            sw = 0;
            pw ^= 1u;
          }
          if (++sx == BST) {
            sx = 0;
            px ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tfull_bar[slot]);
      }
      tc_commit(drain_bar);
      mbar_wait_drain(drain_bar, 0);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int q = warp & 3;
    uint32_t slot_cnt = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      int e, row0, rows, nt;
      if (!tn_unit(args, u, e, row0, rows, nt)) {
        if (lane == 0 && args.status) atomicOr(args.status, kStatusBadExpert);
        continue;
      }
      const int slot = static_cast<int>(slot_cnt % kSlots);
      const uint32_t use = slot_cnt / kSlots;
      ++slot_cnt;
      if (!mbar_wait(&tfull_bar[slot], use & 1u, abort_flag, args.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(slot * kTnMaxN);
      const int prow0 = args.group_padded_offsets[e] + row0;  // stacked row of the chunk's first token
      if (MODE == kStage1) {
        OutT* U = reinterpret_cast<OutT*>(args.U);
        // gate lanes 0-7 and 16-23 hold features f0 .. f0 + 7 and f0 + 8 .. f0 + 15; lanes 0 and 16
        // gather their group's eight results into one 16-byte store per token
        const bool lead_lane = (lane & 15) == 0;
        const bool gate_lane = (lane & 8) == 0;
        const int f = nt * 64 + 16 * q + 8 * (lane >> 4) + (lane & 7);
        // 8-bit kinds: this lane's weight row scale (its gate or up row of feature f)
        float sb = 1.0f;
        if (Q8 && f < args.N)
          sb = args.b_scale[static_cast<size_t>(e) * args.b_scale_rows + (gate_lane ? 0 : args.b_up_offset) + f];
        for (int c0 = 0; c0 < rows; c0 += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + c0, v);
          // 8-bit kinds: lane l holds the activation scale of token c0 + l
          const float sa_l = (Q8 && c0 + lane < rows) ? args.a_scale[prow0 + c0 + lane] : 1.0f;
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float sa = Q8 ? __shfl_sync(0xffffffffu, sa_l, j) : 1.0f;
            const float mine = Q8 ? acc_f32<Q8>(v[j]) * sa * sb : __uint_as_float(v[j]);
            const float other = __shfl_xor_sync(0xffffffffu, mine, 8);
            const float h = silu_mul(mine, other);  // meaningful on the gate lanes
            if (Q8 && args.row_amax) {  // per stacked row amax of U over this warp's 16 features
              // of the value as stored (rounded to OutT), which the quantiser then reads
              float m = (gate_lane && f < args.N) ? fabsf(Elt<OutT>::round(h)) : 0.0f;
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
              if (lane == 0 && c0 + j < rows)
                atomicMax(reinterpret_cast<int*>(args.row_amax) + prow0 + c0 + j, __float_as_int(m));
            }
            const float h1 = __shfl_down_sync(0xffffffffu, h, 1);
            const uint32_t pk0 = Elt<OutT>::pack2(h, h1);
            const uint32_t pk1 = __shfl_down_sync(0xffffffffu, pk0, 2);
            const uint32_t pk2 = __shfl_down_sync(0xffffffffu, pk0, 4);
            const uint32_t pk3 = __shfl_down_sync(0xffffffffu, pk0, 6);
            if (lead_lane && c0 + j < rows && f < args.N) {
              OutT* dst = U + static_cast<size_t>(prow0 + c0 + j) * args.ldu + f;
              if (f + 8 <= args.N) {  // 16-byte aligned: f % 8 == 0 and ldu % 8 == 0
                *reinterpret_cast<uint4*>(dst) = make_uint4(pk0, pk1, pk2, pk3);
              } else {
                const uint32_t pks[4] = {pk0, pk1, pk2, pk3};
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  if (f + i < args.N) dst[i] = reinterpret_cast<const OutT*>(pks)[i];
              }
            }
          }
        }
      } else {
        OutT* out = reinterpret_cast<OutT*>(args.out);
        const int h = nt * kBM + 32 * q + lane;  // output feature of this lane
        const bool lead_lane = (lane & 7) == 0;  // gathers features h .. h + 7 into one 16-byte op
        const float sb = (Q8 && h < args.N) ? args.b_scale[static_cast<size_t>(e) * args.b_scale_rows + h] : 1.0f;
        for (int c0 = 0; c0 < rows; c0 += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + c0, v);
          // lane l looks up token c0 + l's route, destination row and routing weight
          const int p = prow0 + c0 + lane;
          int dst_row = -1;
          float scale = 0.0f;
          if (c0 + lane < rows) {
            if (MODE == kStage2Pad) {
              int route = args.group_offsets[e] + row0 + c0 + lane;
              route = max(0, min(route, args.R - 1));  // reference clamp (SUB/submission.py:935-947)
              scale = load_weight(args.routed, args.routed_dtype, route);
              dst_row = p;
            } else {
              const int route = args.sorted_route_ids[p];
              if (route >= 0 && route < args.R) {
                scale = load_weight(args.routed, args.routed_dtype, route);
                dst_row = route / args.topk;
              }
            }
          }
          if (Q8 && c0 + lane < rows) scale *= args.a_scale[p];  // 8-bit: the token's activation scale
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int row = __shfl_sync(0xffffffffu, dst_row, j);
            const float sc = __shfl_sync(0xffffffffu, scale, j);
            const float mine = (Q8 ? acc_f32<Q8>(v[j]) * sb : __uint_as_float(v[j])) * sc;
            const float next = __shfl_down_sync(0xffffffffu, mine, 1);
            // lane 8g collects the f16x2 pairs of lanes 8g, 8g+2, 8g+4, 8g+6: features h .. h + 7
            const uint32_t pk0 = Elt<OutT>::pack2(mine, next);
            const uint32_t pk1 = __shfl_down_sync(0xffffffffu, pk0, 2);
            const uint32_t pk2 = __shfl_down_sync(0xffffffffu, pk0, 4);
            const uint32_t pk3 = __shfl_down_sync(0xffffffffu, pk0, 6);
            if (row >= 0 && lead_lane && h < args.N) {
              OutT* dst = out + static_cast<size_t>(row) * args.ldo + h;
              if (h + 8 <= args.N) {  // 16-byte aligned: h % 8 == 0 and ldo % 8 == 0
                const uint4 val = make_uint4(pk0, pk1, pk2, pk3);
                if (MODE == kStage2Pad)
                  *reinterpret_cast<uint4*>(dst) = val;
                else
                  red_add_v4(dst, val);
              } else {  // a tile edge that is not a multiple of 8 features: pairs, then a single
                const uint32_t pks[4] = {pk0, pk1, pk2, pk3};
#pragma unroll
                for (int q2 = 0; q2 < 4; ++q2) {
                  const int hh = h + 2 * q2;
                  if (hh + 1 < args.N) {
                    if (MODE == kStage2Pad)
                      *reinterpret_cast<uint32_t*>(dst + 2 * q2) = pks[q2];
                    else
                      red_add_x2(dst + 2 * q2, pks[q2]);
                  } else if (hh < args.N && MODE == kStage2Pad) {
                    dst[2 * q2] = reinterpret_cast<const OutT*>(&pks[q2])[0];  // the pair's low half
                  }
                }
              }
            }
          }
        }
        if (MODE == kStage2Pad) {
          // the expert's padding rows (after its last chunk) are zero in the reference layout
          const int n = args.group_sizes[e];
          if (row0 + rows == n && h < args.N) {
            const int pad_end = args.group_padded_offsets[e + 1];
            for (int r = args.group_padded_offsets[e] + n; r < pad_end; ++r) {
              if constexpr (Elt<OutT>::kBF16)
                out[static_cast<size_t>(r) * args.ldo + h] = __float2bfloat16_rn(0.0f);
              else
                out[static_cast<size_t>(r) * args.ldo + h] = __float2half_rn(0.0f);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[slot]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Entries (expert, token chunk) in expert order: for the ceil(n_e / 256) chunks c of every expert
// with n_e routed rows, entries[2 (base_e + c)] = e and entries[2 (base_e + c) + 1] = base_e; at
// most max_entries are written.
__global__ void __launch_bounds__(1024)
    build_tn_entries_kernel(const int32_t* __restrict__ group_sizes, int E, int max_entries,
                            int32_t* __restrict__ entries, int32_t* __restrict__ n_entries_out) {
  __shared__ int s_warp[32];
  __shared__ int s_base;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (tid == 0) s_base = 0;
  __syncthreads();
  for (int e0 = 0; e0 < E; e0 += blockDim.x) {
    const int e = e0 + tid;
    int chunks = 0, cs = 0;
    if (e < E) tn_chunking(max(group_sizes[e], 0), chunks, cs);
    int incl = chunks;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) s_warp[w] = incl;
    __syncthreads();
    if (w == 0) {
      int v = s_warp[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += x;
      }
      s_warp[lane] = v;
    }
    __syncthreads();
    const int base = s_base + incl - chunks + (w > 0 ? s_warp[w - 1] : 0);
    for (int c = 0; c < chunks && base + c < max_entries; ++c) {
      entries[2 * (base + c)] = e;
      entries[2 * (base + c) + 1] = base;
    }
    __syncthreads();
    if (tid == 0) s_base += s_warp[31];
    __syncthreads();
  }
  if (tid == 0) *n_entries_out = min(s_base, max_entries);
}

}  // namespace moe
