// moe_gemm_pair.cuh — the grouped expert GEMM on CTA pairs: one tcgen05 MMA (cta_group::2)
// spans the tensor cores, shared memory and TMEM of two SMs.
//
// Why: the single-CTA kernel's work unit is 128 rows x 256 columns per SM, and every k-block
// brings 16 KiB of token rows plus 32 KiB of weight rows into that SM (and the MMAs read them back
// out of shared memory). Measured on B200, the grouped GEMM's speed tracks the bytes each SM moves
// per output more than the TMA box count. A CTA pair computes a 256 x 256 unit (two 128-row
// blocks of one expert) with each SM loading its own 128 token rows and HALF of the 256 weight
// rows: 32 KiB per SM per k-block for the same 128 x 256 outputs per SM, a third less intake,
// and each expert's weight tile crosses L2 -> SM once for both blocks. Each SM keeps its 128 x 256
// accumulator in its own TMEM, so two accumulator slots still fit (the epilogue of one unit
// overlaps the next unit's main loop).
//
// Roles (96 + 32 * EPI threads per CTA, both CTAs of the pair):
//   warp 0 lane 0  B producer: this CTA's half of the unit's weight rows (Stage1: the leader the
//                  128 gate rows, the peer the 128 up rows; Stage2: rows 0-127 / 128-255);
//   warp 6 lane 0  A producer: this CTA's 128-row block (the peer skips groups of one block);
//   warp 1         TMEM (512 columns, allocated for the pair); lane 0 of the LEADER (rank 0)
//                  issues the pair MMAs and commits to both CTAs' barriers;
//   warps 2..5     epilogue of this CTA's block, as in the single-CTA kernel.
// All loads complete on the leader's "full" barriers (the leader arms them with both CTAs'
// bytes); the leader's MMA commits arrive on the "empty" and "accumulator full" barriers of both
// CTAs; both CTAs' epilogues arrive on the leader's "accumulator empty" barriers. Loads carry no
// multicast. Every wait is bounded; the final cluster barrier is reached on every path.
#pragma once
#include "moe_gemm.cuh"

namespace moe {

template <int AST, int BST> struct PairRing {
  static constexpr int kAStageBytes = kABytes;          // this CTA's 128 token rows x 128 B
  static constexpr int kBStageBytes = 128 * kKBytes;    // this CTA's 128 of the unit's 256 weight rows
  static constexpr int kRingBytes = AST * kAStageBytes + BST * kBStageBytes;
  static_assert(kRingBytes <= kRingMax, "ring exceeds shared memory");
  static constexpr int kUnitN = 256;                    // accumulator columns per unit
  static constexpr int kSlots = kTmemCols / kUnitN;     // 2
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kRingBytes + 512 /*barriers*/;
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KiB of shared memory a CTA may opt in to");
};

// Tensor maps: tmA token rows (box 128 rows); tmB0 weight rows (box 128 rows): Stage1 gate rows
// (and up rows at +args.b1_row_offset when tmB1 is the same tensor), Stage2 down rows; tmB1
// Stage1 up rows. Work units = (block group of <= 2 blocks, 256-column tile), from args.groups.
template <int MODE, typename OutT, int Q8, int AST, int BST, int EPI = 4>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(96 + EPI * 32, 1)
    moe_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                         const __grid_constant__ CUtensorMap tmB1, const GemmArgs args) {
  using RingT = PairRing<AST, BST>;
  constexpr int kA = RingT::kAStageBytes;
  constexpr int kB = RingT::kBStageBytes;
  constexpr int kN = RingT::kUnitN;
  constexpr int kSlots = RingT::kSlots;
  // An 8-warp epilogue (EPI = 8: two warps per TMEM lane quadrant) hit bounded-wait timeouts
  // on B200 at the contest shapes (a leader full barrier whose byte count never balanced, seen
  // intermittently); its cause is not known, so the pair kernel runs with 4 epilogue warps only.
  static_assert(EPI == 4, "epilogue warps");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring_b = smem;              // [BST][128 rows x 128 B]
  uint8_t* ring_a = smem + BST * kB;   // [AST][128 rows x 128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + RingT::kRingBytes);
  uint64_t* fullA = bars;                     // [AST] leader's count both CTAs' A bytes
  uint64_t* emptyA = fullA + AST;             // [AST]
  uint64_t* fullB = emptyA + AST;             // [BST] leader's count both CTAs' B bytes
  uint64_t* emptyB = fullB + BST;             // [BST]
  uint64_t* tfull_bar = emptyB + BST;         // [kSlots]
  uint64_t* tempty_bar = tfull_bar + kSlots;  // [kSlots] leader's: EPI epilogue warps x 2 CTAs
  uint64_t* drain_bar = tempty_bar + kSlots;  // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(cluster_id_x());
  const int npairs = static_cast<int>(cluster_count_x());

  if (threadIdx.x == 0) {
    for (int s = 0; s < AST; ++s) {
      mbar_init(&fullA[s], 1);
      mbar_init(&emptyA[s], 1);
    }
    for (int s = 0; s < BST; ++s) {
      mbar_init(&fullB[s], 1);
      mbar_init(&emptyB[s], 1);
    }
    for (int a = 0; a < kSlots; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * EPI);
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
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM address published
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int ngroups = args.ngroups >= 0 ? args.ngroups : *args.ngroups_dev;
  const int num_tiles = ngroups * args.n_tiles;
  const int num_kb = (args.K * (Q8 ? 1 : 2) + kKBytes - 1) / kKBytes;
  constexpr int kKElems = Q8 ? kKBytes : kKBytes / 2;

  if (warp == 0 || warp == 6) {
    // ---------------------------------------------------------------- producers
    if (lane == 0) {
      const bool is_b = warp == 0;
      const int depth = is_b ? BST : AST;
      uint64_t* full = is_b ? fullB : fullA;
      uint64_t* empty = is_b ? emptyB : emptyA;
      uint8_t* ring = is_b ? ring_b : ring_a;
      const int stage_bytes = is_b ? kB : kA;
      const uint64_t pol = is_b ? (args.b_evict_first ? l2_policy_evict_first() : l2_policy_evict_normal())
                                : l2_policy_evict_last();
      const CUtensorMap* map = is_b ? ((MODE == kStage1 && !leader) ? &tmB1 : &tmB0) : &tmA;
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      int par[AST > BST ? AST : BST];
#pragma unroll
      for (int s = 0; s < (AST > BST ? AST : BST); ++s) par[s] = -1;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        int fb, nb, nt, e;
        if (!tile_unit<2>(args, tile, fb, nb, nt, e)) continue;
        int row;
        bool load = true;
        uint32_t leader_bytes;
        if (is_b) {
          if (MODE == kStage1)
            row = e * args.b_rows_per_expert + nt * (kN / 2) + (leader ? 0 : args.b1_row_offset);
          else
            row = e * args.b_rows_per_expert + nt * kN + static_cast<int>(rank) * 128;
          leader_bytes = 2u * kB;
        } else {
          load = leader || nb == 2;  // the peer has no block in a one-block group
          row = (fb + static_cast<int>(rank)) * kBM;
          leader_bytes = static_cast<uint32_t>(nb * kA);
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          // The peer waits on every stage too, so both CTAs step through the same phases.
          if (!mbar_wait(&empty[st], ph ^ 1u, abort_flag, args.status)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[st], leader_bytes);
          if (load)
            tma_load_2d_pair(ring + st * stage_bytes, map, mapa_shared(smem_u32(&full[st]), 0), kb * kKElems, row,
                             pol);
          par[st] = static_cast<int>(ph);
          if (++st == depth) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      // Drain: the leader's full barriers count both CTAs' loads; the peer cannot observe its
      // own loads, so on an abort it gives any copy still in flight time to land.
      if (leader) {
        for (int s = 0; s < depth; ++s)
          if (par[s] >= 0) mbar_wait_drain(&full[s], static_cast<uint32_t>(par[s]));
      } else if (!ok) {
        spin_ns(2000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader)
    if (leader && lane == 0) {
      const uint32_t idesc = Q8 == kQF8 ? idesc_f8(2 * kBM, kN)
                             : Q8   ? idesc_i8(2 * kBM, kN)
                                    : idesc_f16(Elt<OutT>::kBF16, 2 * kBM, kN);
      int sa = 0, sb = 0;
      uint32_t pa = 0, pb = 0;
      uint32_t slot_cnt = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        int fb, nb, nt, e;
        if (!tile_unit<2>(args, tile, fb, nb, nt, e)) continue;
        const int slot = static_cast<int>(slot_cnt % kSlots);
        const uint32_t use = slot_cnt / kSlots;
        ++slot_cnt;
        if (!mbar_wait_cluster(&tempty_bar[slot], (use & 1u) ^ 1u, abort_flag, args.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * kN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&fullB[sb], pb, abort_flag, args.status) ||
              !mbar_wait(&fullA[sa], pa, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(ring_a + sa * kA);
          const uint32_t b_addr = smem_u32(ring_b + sb * kB);
#pragma unroll
          for (int k = 0; k < kKBytes / 32; ++k) {
            const uint64_t ad = smem_desc_sw128(a_addr + k * 32);
            const uint64_t bd = smem_desc_sw128(b_addr + k * 32);
            if (Q8 == kQF8)
              mma_f8_pair(d_tmem, ad, bd, idesc, (kb | k) != 0);
            else if (Q8)
              mma_i8_pair(d_tmem, ad, bd, idesc, (kb | k) != 0);
            else
              mma_f16_pair(d_tmem, ad, bd, idesc, (kb | k) != 0);
          }
          tc_commit_pair(&emptyA[sa], 0x3);  // both CTAs' slots are free once the MMAs read them
          tc_commit_pair(&emptyB[sb], 0x3);
          if (++sa == AST) {
            sa = 0;
            pa ^= 1u;
          }
          if (++sb == BST) {
            sb = 0;
            pb ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair(&tfull_bar[slot], 0x3);  // both CTAs' accumulators are ready
      }
      tc_commit_pair(drain_bar, 0x1);
      mbar_wait_drain(drain_bar, 0);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5, 7..10)
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    const int eg = warp >= 7 ? 1 : 0;  // column half (8 epilogue warps)
    constexpr int kCols = MODE == kStage1 ? kN / 2 : kN;
    constexpr int kSpan = kCols / (EPI / 4);
    constexpr int kPassMax = (Q8 && MODE != kStage1) ? 32 : 128;  // as in moe_gemm_kernel
    constexpr int kPass = kSpan < kPassMax ? kSpan : kPassMax;     // columns held in registers per pass
    uint32_t slot_cnt = 0;
    bool ok = true;
    for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
      int fb, nb, nt, e;
      if (!tile_unit<2>(args, tile, fb, nb, nt, e)) {
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
      // hands the slot back to the leader's MMA warp once this warp's TMEM reads are complete
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty_bar[slot]), 0));
      };
      auto keep = []() {};
      if (leader || nb == 2) {
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(slot * kN);
#pragma unroll 1
        for (int c0 = 0; c0 < kSpan; c0 += kPass) {
          if (c0 + kPass < kSpan)
            epilogue_block<MODE, OutT, Q8, kN, kATma, kPass>(args, t_row, fb + static_cast<int>(rank), nt, e,
                                                             row_in_tile, eg * kSpan + c0, keep);
          else
            epilogue_block<MODE, OutT, Q8, kN, kATma, kPass>(args, t_row, fb + static_cast<int>(rank), nt, e,
                                                             row_in_tile, eg * kSpan + c0, release);
        }
      } else {
        release();
      }
    }
  }

  if (MODE == kStage2Comb && args.out_regions != nullptr) __threadfence_system();  // push combine
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its pair may still touch its shared memory or TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace moe
