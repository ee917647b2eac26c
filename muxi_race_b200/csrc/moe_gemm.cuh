// moe_gemm.cuh — the grouped expert GEMM of the fused MoE, as one persistent,
// warp-specialised tcgen05 kernel template for sm_100a.
//
// One CTA per SM (224 threads, 7 warps):
//   warp 0      lane 0 streams B (expert weight rows) into the B ring by TMA;
//   warp 6      streams A (token rows) into the A ring: lane 0 by TMA, or all lanes by cp.async
//               (LSU paths); A and B have separate rings, depths and barriers, so the weight
//               stream never waits for an A slot;
//   warp 1      owns TMEM (512 columns of fp32/int32 accumulators); one lane issues tcgen05.mma
//               for each k-block and commits to the rings' "empty" barriers;
//   warps 2..5  epilogue: tcgen05.ld a finished accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31 = tile rows), apply the fused epilogue, store to global, and hand
//               the slot back, so epilogues overlap the main loop of the next tile.
//
// Work unit = (block group, column tile). A block group is up to GMAX consecutive 128-row
// routing blocks of ONE expert: every k-block of the expert's weight tile is loaded once and
// multiplied against all the group's A blocks (one accumulator slot per block), so an expert
// with 129..256 routed rows streams its weights from HBM once instead of twice (two units that
// read the same weight tile at different times rarely meet in L2: at ~7 TB/s the 126 MB L2 turns
// over in ~18 us). A two-block group's A rows are contiguous and arrive as one 256-row box.
//
// TMA operations per byte: in a streaming microbenchmark on B200 one CTA completes about one TMA
// box per ~300-350 ns almost whatever its size (16 KiB boxes: ~48 GB/s per SM from L2; 64 KiB
// boxes: ~160 GB/s), so the kernel can move fewer, larger boxes: the gate and up rows of a Stage1
// weight tile come as one box of a 3-D/4-D tensor map (the gate/up offset is a tensor dimension),
// and a weight box may span KPB consecutive k-blocks (a k-block dimension of stride 128 bytes),
// which lands in shared memory exactly as KPB consecutive 128B-swizzled k-block tiles. (In the
// full GEMM neither measured faster on cfg3, where the MMA side sets the pace; KPB > 1 stays an
// option.)
//
// CTAs per SM (CPS): with CPS = 2 each CTA takes half the shared memory and half of TMEM, and the
// two CTAs' epilogues and main loops overlap each other.
//
// Tiles: 128 rows per block x BN accumulator columns (BN = 128 or 256: one N = BN MMA per k-step;
// BN = 512: two N = 256 MMAs per k-step sharing the A block). Accumulator slots = 512 / BN, a
// group takes one per block. k-blocks are 128 bytes wide (64 fp16/bf16 or 128 int8 elements,
// 128-byte swizzle): measured on B200, halving the k-block width costs 20% or more.
//
// Modes (the epilogue is the only difference):
//   kStage1     D = [gate | up] halves of BN/2 columns each; U = silu(gate) * up, stored to the
//               [rows, I] intermediate (reference Stage1, SUB/submission.py:586-641);
//   kStage2Pad  out[p, :] = D * routed[route(p)] for valid rows and 0 for pad rows, in the
//               padded stacked layout (reference Stage2, SUB/submission.py:317-357, 933-947);
//   kStage2Comb out[token(p), :] += D * topk_weight(p) via vector red.add into the token-major
//               output (the top-k combine fused into the down GEMM's epilogue).
// 8-bit variants (Q8 = kQI8: int8 with int32 accumulation; kQF8: fp8 e4m3 with fp32
// accumulation) dequantise the accumulator with per-row (token) and per-column (weight output
// row) scales before the same epilogue.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sm100_ptx.cuh"

namespace moe {

constexpr int kBM = 128;       // rows per block = routing block size
constexpr int kMmaN = 256;     // N of one tcgen05.mma
constexpr int kKBytes = 128;   // k-block width in bytes (one 128B swizzle atom)
constexpr int kThreads = 224;  // 7 warps (4 epilogue warps); kernels with 8 epilogue warps use 352
constexpr int kABytes = kBM * kKBytes;  // 16 KiB per A block per stage
constexpr int kTmemCols = 512;
constexpr int kRingMax = 224 * 1024;

// Shared-memory rings: A (token rows, mostly L2 hits) and B (expert weights, streamed from HBM)
// have separate depths, so the weight stream can run further ahead than the A stream. An A stage
// holds one k-block of every block of a group (or, with KPA > 1, KPA k-blocks of one block,
// [k-block][128 rows]); a B stage holds KPB k-blocks of the weight tile, laid out
// [k-block][BN rows] (Stage1 rows: [gate BN/2 | up BN/2]).
template <int BN, int GMAX, int AST, int BST, int CPS = 1, bool ROWTAB = false, int KPB = 1, int KPA = 1>
struct Ring {
  static_assert(BN == 128 || BN == 256 || BN == 512, "accumulator width");
  static_assert(CPS == 1 || CPS == 2, "CTAs per SM");
  static_assert(KPB == 1 || (KPB >= 1 && KPB <= 4 && BN <= kMmaN), "k-blocks per weight box");
  // k-blocks per A box (one 3-D box of KPA consecutive k-blocks of one block's rows): one-block
  // units on the TMA A path only
  static_assert(KPA == 1 || (KPA >= 1 && KPA <= 4 && GMAX == 1 && !ROWTAB), "k-blocks per A box");
  static constexpr int kMN = BN < kMmaN ? BN : kMmaN;  // N of one MMA
  static constexpr int kTmemColsCta = kTmemCols / CPS;  // TMEM columns this CTA allocates
  static_assert(GMAX >= 1 && GMAX * BN <= kTmemColsCta, "a block group must fit in TMEM");
  static constexpr int kAStageBytes = KPA * GMAX * kABytes;
  static constexpr int kBKBytes = BN * kKBytes;  // one k-block of the weight tile
  static constexpr int kBBytes = KPB * kBKBytes;
  static constexpr int kAStages = AST;
  static constexpr int kBStages = BST;
  static constexpr int kRingBytes = AST * kAStageBytes + BST * kBBytes;
  static_assert(kRingBytes <= kRingMax, "ring exceeds shared memory");
  static constexpr int kSlots = kTmemColsCta / BN;  // accumulator slots
  static constexpr int kRowTabBytes = ROWTAB ? GMAX * 128 * 8 : 0;  // LSU A path: source row offsets
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kRingBytes + 512 /*control block*/ + kRowTabBytes;
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KiB of shared memory a CTA may opt in to");
  static_assert(CPS == 1 || kSmemBytes + 1024 <= 233472 / 2, "two CTAs must fit in one SM's shared memory");
};

enum GemmMode : int { kStage1 = 0, kStage2Pad = 1, kStage2Comb = 2 };

struct GemmArgs {
  int K;                      // reduction length in elements
  int N;                      // valid output columns per expert (I for Stage1, H for Stage2)
  int n_tiles;                // column tiles per block group
  int ngroups;                // block groups, or -1: read *ngroups_dev (device-resident count)
  const int* ngroups_dev;
  const int* groups;          // [ngroups] first_block * 2 + (blocks - 1); NULL: group g = block g
  int E;
  const int* block_expert;    // expert of each 128-row block (group_idx_for_bx)
  int nblk;                   // 128-row blocks in the A / output row space (units beyond it are skipped)
  int b_rows_per_expert;      // rows of one expert in the B tensor map(s)
  int b1_row_offset;          // Stage1: row offset of the "up" half inside one expert of map B1

  // Stage1 output: U [rows, ldu]
  void* U;
  int ldu;

  // Stage2 output: out [rows or tokens, ldo]
  void* out;
  int ldo;
  // Stage2Comb into other GPUs' memory (expert parallelism, push combine): the row of virtual
  // route r = (s * out_T_max + t) * topk + j is stored (not added) into row t * topk + j of
  // (OutT*)(out_regions[s] + out_region_off), a per-route slot of token t's home rank s, which
  // sums its token's slots after the exchange; NULL: out
  const uint64_t* out_regions;
  long long out_region_off;
  int out_T_max;
  // Stage2Pad: reference metadata and routed weights
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

  // A operand through the LSU path (kALsu / kAGather): rows of a_row_bytes bytes at a_ptr
  const void* a_ptr;
  long long a_row_bytes;
  // Stage1 with kAGather: the epilogue warps first zero this buffer (the Stage2 combine target)
  void* zero_ptr;
  long long zero_bytes;

  int b_evict_first;          // weight loads with the L2 evict_first policy
  int out_evict_last;         // Stage2Comb: the combine's adds with the L2 evict_last policy
  int unit_order;             // 0 = group-major units, 1 = per expert column-tile-major (tile_unit)
  // Stage1 weight maps: 0 = tmB0 covers gate and up rows as one tensor (the gate/up offset is a
  // dimension: one box per stage); 1 = tmB0 gate rows and tmB1 up rows, two 2-D boxes per k-block.
  int b_split;
  int gu_swap;                // combined map based at the up rows: the tile holds [up | gate]
  int late_release;           // epilogue hands the accumulator slot back after its stores (A/B switch)
  int m64_tail;               // blocks with at most 64 valid rows run M = 64 MMAs (needs group_sizes)

  // Single-kernel MoE (moe_single_kernel): per 128-row block, a count of Stage1 results. Each
  // Stage1 epilogue warp adds one per column tile after its stores of the block's U rows;
  // Stage2's A producer waits until a block's count reaches block_done_target before it loads
  // those rows. NULL: the stages are separate launches and nothing is counted.
  uint32_t* block_done;
  uint32_t block_done_target;

  // Stage1 with gather warps (expert parallelism over peer memory, the fused token gather): the
  // kernel's GW extra warps copy the token row of every routed padded row p, in row order, into
  // row p of g_rows (the A rows): virtual route sorted_route_ids[p] = (s * g_T_max + t) * topk + j
  // names row t of rank s's hidden states, at g_regions[s] + g_x_off. After each row (padding rows
  // too) a warp adds one to a_done[p / 128]; the A producer loads a block once its count reaches
  // 128. A token's row is read once per rank: the warp that claims the token (g_claim[tok], zero
  // at the start of a call) stores it into all its local rows (g_route_slot[tok * topk + j]). With
  // g_zero_y they then zero row tok of g_zero_y (the pull combine's partial rows) for every token
  // tok < g_tokens with a local route.
  const uint64_t* g_regions;
  long long g_x_off;
  int g_T_max;
  void* g_rows;
  uint32_t* a_done;
  void* g_zero_y;
  const int32_t* g_route_slot;
  int g_tokens;
  uint32_t* g_claim;

  uint32_t* status;           // device status word (OR of kStatus* bits)
};

// How the A operand reaches shared memory:
//   kATma        one TMA box per block (rows = padded rows of the A tensor map)
//   kALsu        cp.async by a producer warp, row p of a_ptr
//   kAGather     cp.async by a producer warp, row sorted_route_ids[p] / topk of a_ptr: each routed
//                row reads its token row directly (no stacked copy); padding rows are zero-filled
//   kATmaGather  TMA tile::gather4 loads from a tensor map over the token rows: lane l of the
//                producer warp fetches padded rows 4l..4l+3 of a block (token rows
//                sorted_route_ids[p] / topk; padding rows read token row 0, whose products are
//                never stored), 32 loads per block and k-block; no stacked copy, and the rows of
//                a 128-row block land in the same 128B-swizzled tile as one TMA box would give
// The LSU warp maps 8 lanes to the eight 16-byte chunks of one 128-byte row segment, so every
// instruction moves four whole segments; it is a second load path next to the TMA unit.
enum AMode : int { kATma = 0, kALsu = 1, kAGather = 2, kATmaGather = 3 };

// A modes whose producer writes shared memory with cp.async (generic proxy) and a row table
__host__ __device__ constexpr bool a_mode_lsu(int amode) { return amode == kALsu || amode == kAGather; }

// Source row of padded row p for the A operand, -1 for padding.
template <int AMODE>
__device__ __forceinline__ long long a_source_row(const GemmArgs& args, int p) {
  if (AMODE == kAGather || AMODE == kATmaGather) {
    const int route = args.sorted_route_ids[p];
    return (route >= 0 && route < args.R) ? static_cast<long long>(route / args.topk) : -1;
  }
  return p;
}

// ------------------------------------------------------------------ element helpers
template <typename T> struct Elt;
template <> struct Elt<__half> {
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  // max(|lo|, |hi|) of a packed pair, in fp32
  static __device__ __forceinline__ float amax2(uint32_t v) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&v));
    return fmaxf(fabsf(f.x), fabsf(f.y));
  }
  static __device__ __forceinline__ float round(float a) { return __half2float(__float2half_rn(a)); }
  static constexpr bool kBF16 = false;
};
template <> struct Elt<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float amax2(uint32_t v) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
    return fmaxf(fabsf(f.x), fabsf(f.y));
  }
  static __device__ __forceinline__ float round(float a) { return __bfloat162float(__float2bfloat16_rn(a)); }
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

// The same adds with an L2 cache policy (the combine's target rows kept with evict_last).
__device__ __forceinline__ void red_add_v4(__half* p, uint4 v, uint64_t pol) {
  asm volatile("red.global.add.L2::cache_hint.noftz.v4.f16x2 [%0], {%1,%2,%3,%4}, %5;" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void red_add_v4(__nv_bfloat16* p, uint4 v, uint64_t pol) {
  asm volatile("red.global.add.L2::cache_hint.noftz.v4.bf16x2 [%0], {%1,%2,%3,%4}, %5;" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w), "l"(pol)
               : "memory");
}

__device__ __forceinline__ float load_weight(const void* w, int dtype, int i) {
  if (dtype == 0) return reinterpret_cast<const float*>(w)[i];
  if (dtype == 1) return __half2float(reinterpret_cast<const __half*>(w)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[i]);
}

// Accumulator word -> fp32: int32 for the int8 kind, fp32 otherwise.
template <int Q8>
__device__ __forceinline__ float acc_f32(uint32_t d) {
  if constexpr (Q8 == kQI8) return static_cast<float>(static_cast<int>(d));
  return __uint_as_float(d);
}

// silu(g) * u = g / (1 + e^-g) * u; the exponential is CUDA's __expf.
__device__ __forceinline__ float silu_mul(float g, float u) { return g * __frcp_rn(1.0f + __expf(-g)) * u; }

// Work unit decode: first block, block count, column tile and expert of unit `tile`.
// Units are numbered group-major (n_tiles column tiles per group), so a unit's group g0 names its
// expert. With args.unit_order == 1 the units of one expert are re-ordered column-tile-major:
// for each column tile, all of the expert's groups in turn. The groups of an expert then read the
// same weight tile at the same time on neighbouring SMs, so its second and later reads hit L2
// instead of DRAM. The expert's groups are consecutive, all but the last with gm blocks, so the
// expert's first group is g0 - (first block of g0 - first block of the expert) / gm. Units whose
// blocks fall outside [0, nblk) (metadata inconsistent with the row count) are skipped.
template <int GMAX>
__device__ __forceinline__ bool tile_unit(const GemmArgs& args, int tile, int& fb, int& nb, int& nt, int& e) {
  const int g0 = tile / args.n_tiles;
  const bool grouped = GMAX > 1 && args.groups != nullptr;
  const int pk = grouped ? args.groups[g0] : 0;
  const int fb0 = grouped ? (pk >> 1) : g0;
  e = args.block_expert[fb0];
  if (e < 0 || e >= args.E) return false;
  if (!args.unit_order) {
    nt = tile - g0 * args.n_tiles;
    fb = fb0;
    nb = grouped ? (pk & 1) + 1 : 1;
    return fb >= 0 && fb + nb <= args.nblk;
  }
  const int gm = grouped ? GMAX : 1;
  const int b0 = args.group_padded_offsets[e] / kBM;
  const int nbe = args.group_padded_offsets[e + 1] / kBM - b0;
  const int ng = (nbe + gm - 1) / gm;
  const int gs = g0 - (fb0 - b0) / gm;
  const int local = tile - gs * args.n_tiles;
  if (nbe < 1 || local < 0 || local >= ng * args.n_tiles) return false;  // metadata inconsistent with gidx
  nt = local / ng;
  const int j = local - nt * ng;
  fb = b0 + j * gm;
  nb = min(gm, nbe - j * gm);
  return fb >= 0 && fb + nb <= args.nblk;
}

// An expert's last block with at most 64 valid rows ("half block") runs M = 64 MMAs: half the
// tensor-core work of an M = 128 block. Rows 64..127 of such a block are padding. The M = 64
// accumulator occupies TMEM lanes 0-15 of each 32-lane sub-partition (row r in lane
// r % 16 + 32 * (r / 16)), so epilogue warp q finds rows 16q..16q+15 in its lanes 0-15 and its
// lanes 16-31 hold nothing to store. The padded-store Stage2 (which writes zeros to pad rows)
// keeps M = 128.
template <int MODE>
__device__ __forceinline__ bool half_block(const GemmArgs& args, int e, int mb) {
  if (MODE == kStage2Pad || !args.m64_tail || args.group_sizes == nullptr) return false;
  return args.group_sizes[e] - (mb * kBM - args.group_padded_offsets[e]) <= kBM / 2;
}

// ------------------------------------------------------------------ epilogue of one block
// Columns [c_begin, c_end) of the block's output tile (Stage1: of the BN/2 SiLU*up outputs), in
// chunks of 32: with 8 epilogue warps two warps share a TMEM lane quadrant, each taking half.
//
// Two phases. (1) Every chunk is read from TMEM, finished in registers (dequantisation, SiLU*up
// or the routing weight) and packed to OutT; then `release()` hands the accumulator slot back to
// the MMA warp. (2) The packed values are stored (Stage1 U, Stage2Pad) or added into the output
// (Stage2Comb). The slot is free while the stores and reductions drain, so the next unit's MMAs
// start as soon as the TMEM reads are done: this matters where a unit occupies every slot (a
// two-block group of 256 columns fills all 512 TMEM columns).
template <int MODE, typename OutT, int Q8, int BN, int AMODE, int SPAN, typename Release>
__device__ __forceinline__ void epilogue_block(const GemmArgs& args, uint32_t t_row, int mb, int nt, int e,
                                               int row_in_tile, int c_begin, Release release) {
  static_assert(SPAN % 32 == 0 && SPAN <= 128, "columns per epilogue thread held in registers");
  constexpr int kChunks = SPAN / 32;
  // row_in_tile < 0: this lane reads TMEM with its warp but has no row (lanes 16-31 of a half block)
  const bool has_row = row_in_tile >= 0;
  const int p = mb * kBM + (has_row ? row_in_tile : 0);  // padded row of this thread
  uint32_t packed[kChunks][16];
  if (MODE == kStage1) {
    const int n0 = nt * (BN / 2);
    float sa = 1.0f;
    if (Q8) {
      const long long src = a_source_row<AMODE>(args, p);
      sa = src >= 0 ? args.a_scale[src] : 0.0f;
    }
    float amax = 0.0f;
    const uint32_t goff = args.gu_swap ? BN / 2 : 0;  // [gate | up] or [up | gate] columns
#pragma unroll
    for (int ch = 0; ch < kChunks; ++ch) {
      const int c = c_begin + 32 * ch;
      const int col0 = n0 + c;
      if (col0 >= args.N) continue;  // warp-uniform
      uint32_t g[32], u[32];
      tmem_ld_32x32b_x32(t_row + goff + c, g);
      tmem_ld_32x32b_x32(t_row + (BN / 2 - goff) + c, u);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float g0, g1, u0, u1;
        if (Q8) {
          const int cc = min(col0 + j, args.N - 2);
          const size_t wrow = static_cast<size_t>(e) * args.b_rows_per_expert;
          g0 = acc_f32<Q8>(g[j]) * sa * args.b0_scale[wrow + cc];
          g1 = acc_f32<Q8>(g[j + 1]) * sa * args.b0_scale[wrow + cc + 1];
          u0 = acc_f32<Q8>(u[j]) * sa * args.b1_scale[wrow + args.b1_row_offset + cc];
          u1 = acc_f32<Q8>(u[j + 1]) * sa * args.b1_scale[wrow + args.b1_row_offset + cc + 1];
        } else {
          g0 = __uint_as_float(g[j]);
          g1 = __uint_as_float(g[j + 1]);
          u0 = __uint_as_float(u[j]);
          u1 = __uint_as_float(u[j + 1]);
        }
        packed[ch][j / 2] = Elt<OutT>::pack2(silu_mul(g0, u0), silu_mul(g1, u1));
        // the requantisation scale comes from the values as stored (rounded to OutT), the same
        // values the quantiser then reads
        if (Q8 && col0 + j < args.N) amax = fmaxf(amax, Elt<OutT>::amax2(packed[ch][j / 2]));
      }
    }
    if (!args.late_release) release();
    OutT* U = reinterpret_cast<OutT*>(args.U);
#pragma unroll
    for (int ch = 0; ch < kChunks; ++ch) {
      const int col0 = n0 + c_begin + 32 * ch;
      if (col0 >= args.N || !has_row) continue;
      OutT* dst = U + static_cast<size_t>(p) * args.ldu + col0;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        if (col0 + v * 8 < args.N)
          *reinterpret_cast<uint4*>(dst + v * 8) =
              make_uint4(packed[ch][4 * v], packed[ch][4 * v + 1], packed[ch][4 * v + 2], packed[ch][4 * v + 3]);
      }
    }
    if (Q8 && args.row_amax && has_row) atomicMax(reinterpret_cast<int*>(args.row_amax) + p, __float_as_int(amax));
    if (args.late_release) release();
  } else {
    const int n0 = nt * BN;
    float scale = 0.0f;
    bool valid = false;
    int token = 0;
    int route_id = 0;
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
      valid = has_row && route >= 0 && route < args.R;
      if (valid) {
        token = route / args.topk;
        route_id = route;
        scale = load_weight(args.routed, args.routed_dtype, route);
      }
    }
    float sa = 1.0f;
    if (Q8) sa = args.a_scale[p];
#pragma unroll
    for (int ch = 0; ch < kChunks; ++ch) {
      const int c = c_begin + 32 * ch;
      const int col0 = n0 + c;
      if (col0 >= args.N) continue;  // warp-uniform
      uint32_t d[32];
      tmem_ld_32x32b_x32(t_row + c, d);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float d0, d1;
        if (Q8) {
          const int cc = min(col0 + j, args.N - 2);
          const size_t wrow = static_cast<size_t>(e) * args.b_rows_per_expert;
          d0 = acc_f32<Q8>(d[j]) * sa * args.b0_scale[wrow + cc];
          d1 = acc_f32<Q8>(d[j + 1]) * sa * args.b0_scale[wrow + cc + 1];
        } else {
          d0 = __uint_as_float(d[j]);
          d1 = __uint_as_float(d[j + 1]);
        }
        packed[ch][j / 2] = valid ? Elt<OutT>::pack2(d0 * scale, d1 * scale) : 0u;
      }
    }
    if (!args.late_release) release();
    OutT* out = reinterpret_cast<OutT*>(args.out);
    size_t orow = MODE == kStage2Pad ? static_cast<size_t>(p) : static_cast<size_t>(token);
    const bool push = MODE == kStage2Comb && args.out_regions != nullptr;
    if (push && valid) {  // this route's slot at the token's home rank
      const int home = token / args.out_T_max;
      out = reinterpret_cast<OutT*>(args.out_regions[home] + static_cast<uint64_t>(args.out_region_off));
      orow = static_cast<size_t>(route_id) - static_cast<size_t>(home) * args.out_T_max * args.topk;
    }
#pragma unroll
    for (int ch = 0; ch < kChunks; ++ch) {
      const int col0 = n0 + c_begin + 32 * ch;
      if (col0 >= args.N || (MODE == kStage2Comb && !valid)) continue;
      OutT* dst = out + orow * args.ldo + col0;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        if (col0 + v * 8 >= args.N) continue;
        const uint4 val = make_uint4(packed[ch][4 * v], packed[ch][4 * v + 1], packed[ch][4 * v + 2], packed[ch][4 * v + 3]);
        if (MODE == kStage2Pad || push)
          *reinterpret_cast<uint4*>(dst + v * 8) = val;
        else if (args.out_evict_last)
          red_add_v4(dst + v * 8, val, l2_policy_evict_last());
        else
          red_add_v4(dst + v * 8, val);
      }
    }
    if (args.late_release) release();
  }
}

// ------------------------------------------------------------------ the kernel
// Tensor maps (all 128B-swizzled, boxes 128 bytes wide in k):
//   tmA   A rows, box GMAX * 128 rows: a whole group in one box (TMA A path)
//   tmA1  A rows, box 128 rows: groups with fewer than GMAX blocks (GMAX = 1: the same as tmA)
//   tmB0  weights. Stage1: one map over the gate and up rows (dimensions {K, rows, gate/up} for
//         KPB = 1, {k-block elements, rows, gate/up, k-blocks} otherwise), or the gate rows alone
//         when args.b_split. Stage2: {K, rows} for KPB = 1, {k-block elements, rows, k-blocks}
//         otherwise.
//   tmB1  Stage1 with args.b_split: the up rows ({K, rows}).
// Control block after the rings: the TMEM base address (4 bytes), the abort flag (4 bytes), then
// the mbarriers of one pipeline (two in the single-kernel MoE, one set per stage).
constexpr int kCtlBytes = 512;
__host__ __device__ constexpr int pipeline_bars(int ast, int bst, int slots) { return 2 * ast + 2 * bst + 2 * slots + 1; }

// The roles of one grouped GEMM over its work units, on a CTA whose TMEM is allocated (the
// address is at *tmem_slot once the CTA has synchronised) and whose abort flag is cleared: the
// phase initialises its mbarriers at `bars`, runs the producers, the MMA issuer and the
// epilogue, and returns once every role has drained (its loads landed, its MMAs retired).
template <int MODE, typename OutT, int Q8, int BN, int GMAX, int AST, int BST, int AMODE, int CPS, int KPB, int EPI,
          int KPA = 1, int GW = 0>
__device__ __forceinline__ void gemm_phase(const CUtensorMap* tmA_p, const CUtensorMap* tmA1_p,
                                           const CUtensorMap* tmB0_p, const CUtensorMap* tmB1_p,
                                           const GemmArgs& args, uint8_t* smem, uint64_t* bars,
                                           const uint32_t* tmem_slot, volatile int* abort_flag, long long* row_tab) {
  using RingT = Ring<BN, GMAX, AST, BST, CPS, a_mode_lsu(AMODE), KPB, KPA>;
  static_assert(KPA == 1 || AMODE == kATma, "multi-k-block A boxes are TMA boxes");
  static_assert(GW == 0 || (MODE == kStage1 && AMODE == kATma && GMAX == 1), "gather warps feed one-block Stage1 units");
  constexpr int kAStageBytes = RingT::kAStageBytes;
  constexpr int kBBytes = RingT::kBBytes;
  constexpr int kBKBytes = RingT::kBKBytes;
  constexpr int kMN = RingT::kMN;
  constexpr int kSlots = RingT::kSlots;
  constexpr int kHalves = BN / kMN;  // MMAs per k-step per block
  static_assert(EPI == 4 || EPI == 8, "epilogue warps");
  const CUtensorMap& tmA = *tmA_p;
  const CUtensorMap& tmA1 = *tmA1_p;
  const CUtensorMap& tmB0 = *tmB0_p;
  const CUtensorMap& tmB1 = *tmB1_p;
  uint8_t* ring_b = smem;                            // [BST][KPB][BN rows x 128 B]
  uint8_t* ring_a = smem + BST * kBBytes;            // [AST][GMAX][kABytes]
  uint64_t* fullA = bars;                            // [AST]
  uint64_t* emptyA = fullA + AST;                    // [AST]
  uint64_t* fullB = emptyA + AST;                    // [BST]
  uint64_t* emptyB = fullB + BST;                    // [BST]
  uint64_t* tfull_bar = emptyB + BST;                // [kSlots] per accumulator slot
  uint64_t* tempty_bar = tfull_bar + kSlots;         // [kSlots]
  uint64_t* drain_bar = tempty_bar + kSlots;         // [1] MMA warp: all issued MMAs retired
  auto stage_a = [&](int s, int j) { return ring_a + s * kAStageBytes + j * kABytes; };
  auto stage_b = [&](int s) { return ring_b + s * kBBytes; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < AST; ++s) {
      mbar_init(&fullA[s], a_mode_lsu(AMODE) ? 32 : 1);  // TMA: expect_tx arrive; LSU: one per lane
      mbar_init(&emptyA[s], 1);
    }
    for (int s = 0; s < BST; ++s) {
      mbar_init(&fullB[s], 1);
      mbar_init(&emptyB[s], 1);
    }
    for (int a = 0; a < kSlots; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], EPI);  // one arrive per epilogue warp
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    if (!a_mode_lsu(AMODE)) {
      tma_prefetch_desc(&tmA);
      if (GMAX > 1) tma_prefetch_desc(&tmA1);
    }
    tma_prefetch_desc(&tmB0);
    if (MODE == kStage1 && args.b_split) tma_prefetch_desc(&tmB1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int ngroups = args.ngroups >= 0 ? args.ngroups : *args.ngroups_dev;
  const int num_tiles = ngroups * args.n_tiles;
  const int num_kb = (args.K * (Q8 ? 1 : 2) + kKBytes - 1) / kKBytes;
  constexpr int kKElems = Q8 ? kKBytes : kKBytes / 2;

  if (warp == 0) {
    // ---------------------------------------------------------------- B producer (weights)
    // One lane streams the weight tile of each unit, KPB k-blocks per ring stage, up to BST
    // stages ahead of the MMA. L2 policy evict_normal (args.b_evict_first: evict_first).
    if (lane == 0) {
      const uint64_t pol = args.b_evict_first ? l2_policy_evict_first() : l2_policy_evict_normal();
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      int par[BST];  // parity of the last load issued into each slot, -1 = none
#pragma unroll
      for (int s = 0; s < BST; ++s) par[s] = -1;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int fb, nb, nt, e;
        if (!tile_unit<GMAX>(args, tile, fb, nb, nt, e)) continue;
        const int brow = e * args.b_rows_per_expert + nt * (MODE == kStage1 ? BN / 2 : BN);
        for (int kb0 = 0; kb0 < num_kb; kb0 += KPB) {
          if (!mbar_wait(&emptyB[st], ph ^ 1u, abort_flag, args.status)) {
            ok = false;
            break;
          }
          uint8_t* dst = stage_b(st);
          if (MODE == kStage1 && args.b_split) {  // gate box + up box per k-block
            const int nk = min(KPB, num_kb - kb0);
            mbar_arrive_expect_tx(&fullB[st], static_cast<uint32_t>(nk * kBKBytes));
            for (int j = 0; j < nk; ++j) {
              const int kx = (kb0 + j) * kKElems;
              tma_load_2d(dst + j * kBKBytes, &tmB0, &fullB[st], kx, brow, pol);
              tma_load_2d(dst + j * kBKBytes + kBKBytes / 2, &tmB1, &fullB[st], kx, brow + args.b1_row_offset, pol);
            }
          } else {
            mbar_arrive_expect_tx(&fullB[st], static_cast<uint32_t>(kBBytes));
            if (MODE == kStage1) {  // gate and up rows of KPB k-blocks in one box
              if (KPB == 1)
                tma_load_3d(dst, &tmB0, &fullB[st], kb0 * kKElems, brow, 0, pol);
              else
                tma_load_4d(dst, &tmB0, &fullB[st], 0, brow, 0, kb0, pol);
            } else if (KPB == 1) {
#pragma unroll
              for (int h = 0; h < kHalves; ++h)
                tma_load_2d(dst + h * (kMN * kKBytes), &tmB0, &fullB[st], kb0 * kKElems, brow + h * kMN, pol);
            } else {
              tma_load_3d(dst, &tmB0, &fullB[st], 0, brow, kb0, pol);
            }
          }
          par[st] = static_cast<int>(ph);
          if (++st == BST) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      // Drain: every load issued must have landed before the CTA may exit. On the normal path
      // these phases completed long ago; after an abort this bounds the wait.
      for (int s = 0; s < BST; ++s)
        if (par[s] >= 0) mbar_wait_drain(&fullB[s], static_cast<uint32_t>(par[s]));
    }
  } else if (warp == 6) {
    // ---------------------------------------------------------------- A producer (token rows)
    // TMA from lane 0 (kATma; a full group as one box) or cp.async from all 32 lanes (LSU paths),
    // one k-block per stage, up to AST stages ahead. L2 policy evict_last: every column tile of
    // the group re-reads these rows.
    if (AMODE == kATmaGather) {
      // Every lane: its four padded rows of each block of the unit as token rows, then per
      // k-block lane 0 arms the stage with the group's bytes and each lane issues one gather4 per
      // block (4 rows x 128 bytes at byte 512 * lane of the block's tile). The 128B swizzle is a
      // function of the shared-memory address, so the 32 pieces form the same tile as a 128-row
      // box (the 8-row swizzle atoms are 1024-byte aligned; a piece is half an atom).
      const uint64_t pol = l2_policy_evict_last();
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      int par[AST];
#pragma unroll
      for (int s = 0; s < AST; ++s) par[s] = -1;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int fb, nb, nt, e;
        if (!tile_unit<GMAX>(args, tile, fb, nb, nt, e)) continue;
        int rows[GMAX][4];
#pragma unroll
        for (int j = 0; j < GMAX; ++j)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const long long src = j < nb ? a_source_row<AMODE>(args, (fb + j) * kBM + 4 * lane + i) : -1;
            rows[j][i] = src >= 0 ? static_cast<int>(src) : 0;
          }
        for (int kb = 0; kb < num_kb; ++kb) {
          const bool got = __all_sync(0xffffffffu, mbar_wait(&emptyA[st], ph ^ 1u, abort_flag, args.status));
          if (!got) {
            ok = false;
            break;
          }
          if (lane == 0) mbar_arrive_expect_tx(&fullA[st], static_cast<uint32_t>(nb * kABytes));
          __syncwarp();
          const int kx = kb * kKElems;
#pragma unroll
          for (int j = 0; j < GMAX; ++j)
            if (j < nb)
              tma_gather4(stage_a(st, j) + lane * 4 * kKBytes, &tmA, &fullA[st], kx, rows[j][0], rows[j][1],
                          rows[j][2], rows[j][3], pol);
          par[st] = static_cast<int>(ph);
          if (++st == AST) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      // Drain: a phase completes only when every lane's loads of it have landed
      if (lane == 0)
        for (int s = 0; s < AST; ++s)
          if (par[s] >= 0) mbar_wait_drain(&fullA[s], static_cast<uint32_t>(par[s]));
      __syncwarp();
    } else if (AMODE != kATma || lane == 0) {
      const uint64_t pol = l2_policy_evict_last();
      const long long a_k_bytes = static_cast<long long>(args.K) * (Q8 ? 1 : 2);
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      int par[AST];
#pragma unroll
      for (int s = 0; s < AST; ++s) par[s] = -1;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int fb, nb, nt, e;
        if (!tile_unit<GMAX>(args, tile, fb, nb, nt, e)) continue;
        if (GW > 0 && args.a_done != nullptr) {
          // the gather warps of all CTAs have copied every row of this block (generic-proxy stores
          // read here by TMA: acquire, then the proxy fence)
          bool dep = true;
          for (int j = 0; j < nb && dep; ++j)
            dep = counter_wait(args.a_done + fb + j, static_cast<uint32_t>(kBM), abort_flag, args.status);
          if (!dep) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
        }
        if (MODE != kStage1 && AMODE == kATma && args.block_done != nullptr) {
          // single-kernel MoE: the group's U rows are complete once every Stage1 column tile of
          // each of its blocks has published its stores (other CTAs' generic-proxy stores, read
          // here by TMA: acquire, then the proxy fence)
          bool dep = true;
          for (int j = 0; j < nb && dep; ++j)
            dep = counter_wait(args.block_done + fb + j, args.block_done_target, abort_flag, args.status);
          if (!dep) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
        }
        if (AMODE != kATma) {
          // byte offsets of this group's source rows, -1 = zero fill
          __syncwarp();
          for (int j = 0; j < nb; ++j)
            for (int r = lane; r < kBM; r += 32) {
              const long long src = a_source_row<AMODE>(args, (fb + j) * kBM + r);
              row_tab[j * kBM + r] = src >= 0 ? src * args.a_row_bytes : -1;
            }
          __syncwarp();
        }
        for (int kb = 0; kb < num_kb; kb += KPA) {
          const int kx = kb * kKElems;
          bool got = mbar_wait(&emptyA[st], ph ^ 1u, abort_flag, args.status);
          if (AMODE != kATma) got = __all_sync(0xffffffffu, got);  // the warp stays converged
          if (!got) {
            ok = false;
            break;
          }
          if (AMODE == kATma && KPA > 1) {  // KPA k-blocks of the block's rows in one 3-D box
            mbar_arrive_expect_tx(&fullA[st], static_cast<uint32_t>(KPA * kABytes));
            tma_load_3d(stage_a(st, 0), &tmA, &fullA[st], 0, fb * kBM, kb, pol);
          } else if (AMODE == kATma) {
            mbar_arrive_expect_tx(&fullA[st], static_cast<uint32_t>(nb * kABytes));
            if (GMAX > 1 && nb == GMAX)
              tma_load_2d(stage_a(st, 0), &tmA, &fullA[st], kx, fb * kBM, pol);
            else
              for (int j = 0; j < nb; ++j)
                tma_load_2d(stage_a(st, j), GMAX > 1 ? &tmA1 : &tmA, &fullA[st], kx, (fb + j) * kBM, pol);
          } else {
            const int c = lane & 7;  // 16-byte chunk of the 128-byte k-block row segment
            const long long kbyte = static_cast<long long>(kb) * kKBytes + c * 16;
            const bool k_in = kbyte < a_k_bytes;
            const char* a_base = static_cast<const char*>(args.a_ptr);
            for (int j = 0; j < nb; ++j) {
              const uint32_t dst0 = smem_u32(stage_a(st, j));
#pragma unroll 8
              for (int i = 0; i < kBM / 4; ++i) {
                const int r = (lane >> 3) + 4 * i;
                const long long off = row_tab[j * kBM + r];
                const bool in = k_in && off >= 0;
                // 128-byte swizzle: chunk c of row r sits at chunk c ^ (r % 8)
                cp_async_16(dst0 + r * kKBytes + ((c ^ (r & 7)) << 4), in ? a_base + off + kbyte : a_base,
                            in ? 16u : 0u);
              }
            }
            cp_async_mbar_arrive(&fullA[st]);
            mbar_arrive(&fullA[st]);
          }
          par[st] = static_cast<int>(ph);
          if (++st == AST) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      if (AMODE != kATma) cp_async_wait_all();
      if (AMODE == kATma)
        for (int s = 0; s < AST; ++s)
          if (par[s] >= 0) mbar_wait_drain(&fullA[s], static_cast<uint32_t>(par[s]));
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = Q8 == kQF8 ? idesc_f8(kBM, kMN)
                             : Q8   ? idesc_i8(kBM, kMN)
                                    : idesc_f16(Elt<OutT>::kBF16, kBM, kMN);
      const uint32_t idesc64 = Q8 == kQF8 ? idesc_f8(kBM / 2, kMN)
                               : Q8   ? idesc_i8(kBM / 2, kMN)
                                      : idesc_f16(Elt<OutT>::kBF16, kBM / 2, kMN);
      int sa = 0, sb = 0;
      uint32_t pa = 0, pb = 0;
      uint32_t slot_cnt = 0;  // accumulator slots handed out so far (slot = cnt % kSlots)
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int fb, nb, nt, e;
        if (!tile_unit<GMAX>(args, tile, fb, nb, nt, e)) continue;
        uint32_t d_tmem[GMAX];
        uint32_t id_blk[GMAX];  // M = 128, or M = 64 for a half block
        int slot[GMAX];
#pragma unroll
        for (int j = 0; j < GMAX; ++j) id_blk[j] = (j < nb && half_block<MODE>(args, e, fb + j)) ? idesc64 : idesc;
#pragma unroll
        for (int j = 0; j < GMAX; ++j) {
          if (j >= nb || !ok) break;
          slot[j] = static_cast<int>(slot_cnt % kSlots);
          const uint32_t use = slot_cnt / kSlots;  // times this slot was used before
          if (!mbar_wait(&tempty_bar[slot[j]], (use & 1u) ^ 1u, abort_flag, args.status)) ok = false;
          d_tmem[j] = tmem_base + static_cast<uint32_t>(slot[j] * BN);
          ++slot_cnt;
        }
        if (!ok) break;
        tc_fence_after();
        for (int kb = 0; kb < num_kb; ++kb) {
          const int kk = kb % KPB;  // k-block inside the current B stage
          const int ka = kb % KPA;  // k-block inside the current A stage
          if (kk == 0 && !mbar_wait(&fullB[sb], pb, abort_flag, args.status)) {
            ok = false;
            break;
          }
          if (ka == 0 && !mbar_wait(&fullA[sa], pa, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (a_mode_lsu(AMODE)) fence_proxy_async_smem();  // A arrived through the generic proxy
          const uint32_t b_addr = smem_u32(stage_b(sb)) + static_cast<uint32_t>(kk * kBKBytes);
#pragma unroll
          for (int j = 0; j < GMAX; ++j) {
            if (j >= nb) break;
            const uint32_t a_addr = smem_u32(stage_a(sa, j)) + static_cast<uint32_t>(ka * kABytes);
#pragma unroll
            for (int k = 0; k < kKBytes / 32; ++k) {
              const uint64_t ad = smem_desc_sw128(a_addr + k * 32);
#pragma unroll
              for (int h = 0; h < kHalves; ++h) {
                const uint64_t bd = smem_desc_sw128(b_addr + h * (kMN * kKBytes) + k * 32);
                const uint32_t d = d_tmem[j] + static_cast<uint32_t>(h * kMN);
                if (Q8 == kQF8)
                  mma_f8(d, ad, bd, id_blk[j], (kb | k) != 0);
                else if (Q8)
                  mma_i8(d, ad, bd, id_blk[j], (kb | k) != 0);
                else
                  mma_f16(d, ad, bd, id_blk[j], (kb | k) != 0);
              }
            }
          }
          if (ka == KPA - 1 || kb == num_kb - 1) {  // last k-block of the A stage
            tc_commit(&emptyA[sa]);  // frees the A slot once the MMAs have read it
            if (++sa == AST) {
              sa = 0;
              pa ^= 1u;
            }
          }
          if (kk == KPB - 1 || kb == num_kb - 1) {  // last k-block of the B stage
            tc_commit(&emptyB[sb]);
            if (++sb == BST) {
              sb = 0;
              pb ^= 1u;
            }
          }
        }
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < GMAX; ++j)
          if (j < nb) tc_commit(&tfull_bar[slot[j]]);  // accumulators ready for the epilogue
      }
      // Drain: all MMAs this thread issued retire before TMEM is released.
      tc_commit(drain_bar);
      mbar_wait_drain(drain_bar, 0);
    }
  } else if (GW > 0 && warp >= 3 + EPI) {
    // ---------------------------------------------------------------- gather warps
    // Rows in order, so the blocks the first units need are complete first. Eight 16-byte peer
    // loads in flight per lane (NVLink reads have microseconds of latency). Every row, padding
    // included, adds exactly one to its block's count.
    const int gw = static_cast<int>(blockIdx.x) * GW + (warp - 3 - EPI);
    const int n_gw = static_cast<int>(gridDim.x) * GW;
    const int rows = ngroups * kBM;
    const int vecs = static_cast<int>(args.a_row_bytes / 16);
    char* a_rows = static_cast<char*>(args.g_rows);
    for (int p = gw; p < rows; p += n_gw) {
      const int route = args.sorted_route_ids[p];
      if (route < 0 || route >= args.R) {  // padding row: nothing to copy
        if (lane == 0) atomicAdd(args.a_done + (p >> 7), 1u);
        continue;
      }
      // The first warp to reach one of a token's rows claims the token, reads its row over NVLink
      // once and stores it into all the token's local rows (a token's lowest row comes first in
      // row order, so every row of a block is claimed by the time the block's rows are passed).
      const long long tok = route / args.topk;
      int claimed = 0;
      if (lane == 0) claimed = atomicCAS(reinterpret_cast<int*>(args.g_claim) + tok, 0, 1) == 0;
      if (!__shfl_sync(0xffffffffu, claimed, 0)) continue;
      const int my_slot = lane < args.topk ? args.g_route_slot[tok * args.topk + lane] : -1;
      const unsigned local = __ballot_sync(0xffffffffu, my_slot >= 0);
      const int s = static_cast<int>(tok / args.g_T_max);
      const long long t = tok - static_cast<long long>(s) * args.g_T_max;
      const uint4* src =
          reinterpret_cast<const uint4*>(args.g_regions[s] + static_cast<uint64_t>(args.g_x_off)) + t * vecs;
      constexpr int U = 8;
      for (int v0 = lane; v0 < vecs; v0 += 32 * U) {
        uint4 tmp[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (v0 + u * 32 < vecs) tmp[u] = __ldcg(src + v0 + u * 32);
        for (unsigned m = local; m != 0u; m &= m - 1u) {
          const int q = __shfl_sync(0xffffffffu, my_slot, __ffs(static_cast<int>(m)) - 1);
          uint4* dst = reinterpret_cast<uint4*>(a_rows + static_cast<size_t>(q) * args.a_row_bytes);
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (v0 + u * 32 < vecs) dst[v0 + u * 32] = tmp[u];
        }
      }
      fence_proxy_async_global();
      __threadfence();
      __syncwarp();
      if (my_slot >= 0) atomicAdd(args.a_done + (my_slot >> 7), 1u);  // one per row stored
    }
    if (args.g_zero_y != nullptr) {
      uint4* y = static_cast<uint4*>(args.g_zero_y);
      for (int tok = gw; tok < args.g_tokens; tok += n_gw) {
        const int slot = lane < args.topk ? args.g_route_slot[static_cast<long long>(tok) * args.topk + lane] : -1;
        if (__ballot_sync(0xffffffffu, slot >= 0) == 0u) continue;
        uint4* dst = y + static_cast<long long>(tok) * vecs;
        for (int v = lane; v < vecs; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5, 7..10)
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = q * 32 + lane;
    const int eg = warp >= 7 ? 1 : 0;  // column half (8 epilogue warps)
    constexpr int kCols = MODE == kStage1 ? BN / 2 : BN;
    constexpr int kSpan = kCols / (EPI / 4);
    // columns a thread finishes per block; wider spans (BN = 512, or Stage2 BN = 256 with 4
    // epilogue warps) are done in passes of 128 columns, the slot released after the last pass
    // (32 for the 8-bit Stage2, whose per-column dequantisation needs the registers)
    constexpr int kPassMax = (Q8 && MODE != kStage1) ? 32 : 128;
    constexpr int kPass = kSpan < kPassMax ? kSpan : kPassMax;
    const int c_begin = eg * kSpan;
    if (MODE == kStage1 && args.zero_ptr != nullptr) {
      // clear the Stage2 combine target while the first tile's main loop runs
      uint4* z = static_cast<uint4*>(args.zero_ptr);
      const long long n16 = args.zero_bytes / 16;
      const int et = eg * 128 + (warp - (eg ? 7 : 2)) * 32 + lane;
      const long long t0 = static_cast<long long>(blockIdx.x) * (EPI * 32) + et;
      for (long long i2 = t0; i2 < n16; i2 += static_cast<long long>(gridDim.x) * (EPI * 32))
        z[i2] = make_uint4(0, 0, 0, 0);
    }
    uint32_t slot_cnt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int fb, nb, nt, e;
      if (!tile_unit<GMAX>(args, tile, fb, nb, nt, e)) {
        if (lane == 0 && args.status) atomicOr(args.status, kStatusBadExpert);
        continue;
      }
      for (int j = 0; j < nb; ++j) {
        const int slot = static_cast<int>(slot_cnt % kSlots);
        const uint32_t use = slot_cnt / kSlots;
        if (!mbar_wait(&tfull_bar[slot], use & 1u, abort_flag, args.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t_row =
            tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(slot * BN);
        // hands the slot back to the MMA warp once this warp's TMEM reads of it are complete
        auto release = [&]() {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty_bar[slot]);
        };
        auto keep = []() {};
        // a half block's rows 16q..16q+15 sit in lanes 0-15 of quadrant q
        const int row = half_block<MODE>(args, e, fb + j) ? (lane < 16 ? 16 * q + lane : -1) : row_in_tile;
#pragma unroll 1
        for (int c0 = 0; c0 < kSpan; c0 += kPass) {
          if (c0 + kPass < kSpan)
            epilogue_block<MODE, OutT, Q8, BN, AMODE, kPass>(args, t_row, fb + j, nt, e, row, c_begin + c0, keep);
          else
            epilogue_block<MODE, OutT, Q8, BN, AMODE, kPass>(args, t_row, fb + j, nt, e, row, c_begin + c0, release);
        }
        if (MODE == kStage1 && args.block_done != nullptr) {
          // publish this warp's U stores of the block to the Stage2 TMA loads of any CTA
          fence_proxy_async_global();
          __threadfence();
          __syncwarp();
          if (lane == 0) atomicAdd(args.block_done + fb + j, 1u);
        }
        ++slot_cnt;
      }
    }
  }

}

// One grouped GEMM (one stage) per launch.
template <int MODE, typename OutT, int Q8, int BN, int GMAX, int AST, int BST, int AMODE, int CPS, int KPB,
          int EPI = 4, int KPA = 1, int GW = 0>
__global__ void __launch_bounds__(96 + EPI * 32 + GW * 32, CPS)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA1,
                    const __grid_constant__ CUtensorMap tmB0, const __grid_constant__ CUtensorMap tmB1,
                    const GemmArgs args) {
  using RingT = Ring<BN, GMAX, AST, BST, CPS, a_mode_lsu(AMODE), KPB, KPA>;
  static_assert(8 + 8 * pipeline_bars(AST, BST, RingT::kSlots) <= kCtlBytes, "control block");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ctl = smem + RingT::kRingBytes;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctl + 4);
  uint64_t* bars = reinterpret_cast<uint64_t*>(ctl + 8);
  long long* row_tab = reinterpret_cast<long long*>(ctl + kCtlBytes);  // [GMAX][128], LSU A paths
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) *abort_flag = 0;
  if (warp == 1) {
    tmem_alloc(tmem_slot, RingT::kTmemColsCta);
    tmem_relinquish();
  }
  gemm_phase<MODE, OutT, Q8, BN, GMAX, AST, BST, AMODE, CPS, KPB, EPI, KPA, GW>(&tmA, &tmA1, &tmB0, &tmB1, args,
                                                                                 smem, bars, tmem_slot, abort_flag,
                                                                                 row_tab);
  // push combine: this thread's reductions into peer memory are performed system-wide before
  // the kernel ends (the flag barrier that follows publishes them to the home ranks)
  if (MODE == kStage2Comb && args.out_regions != nullptr) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(*tmem_slot, RingT::kTmemColsCta);
  }
}

// ------------------------------------------------------------------ single-kernel MoE
// Stage1 and Stage2 in one persistent launch (one CTA per SM, all co-resident: the launch is
// cooperative). Each CTA runs its Stage1 units (tile 256a4b5e8: 128 SiLU*up columns per unit),
// then, without waiting for the other CTAs, its Stage2 units (tile 256x2a3b4e8: two-block groups,
// 256 output columns). A Stage2 unit loads a block's U rows only after every Stage1 column tile of
// that block has published its stores (GemmArgs::block_done, counted per epilogue warp), so the
// end of Stage1 on one SM overlaps Stage2 on the others: the separate launches' Stage1 tail, launch
// gap and Stage2 prologue are gone; U still goes through memory. Every Stage1 unit is taken before
// any Stage2 unit and Stage1 units wait on nothing outside their CTA, so the waits end as long as
// all CTAs run at once (a cooperative launch guarantees it; each wait is bounded all the same).
// The two phases keep separate mbarriers: asynchronous arrivals of the first can never meet the
// second.
using SingleRing1 = Ring<256, 1, 4, 5>;
using SingleRing2 = Ring<256, 2, 3, 4>;
constexpr int kSingleRingBytes =
    SingleRing1::kRingBytes > SingleRing2::kRingBytes ? SingleRing1::kRingBytes : SingleRing2::kRingBytes;
constexpr int kSingleBars1 = pipeline_bars(4, 5, SingleRing1::kSlots);
constexpr int kSingleBars2 = pipeline_bars(3, 4, SingleRing2::kSlots);
static_assert(8 + 8 * (kSingleBars1 + kSingleBars2) <= kCtlBytes, "control block of the single kernel");
constexpr int kSingleSmemBytes = 1024 + kSingleRingBytes + kCtlBytes;
constexpr int kSingleThreads = 96 + 8 * 32;

template <typename OutT, int MODE2>
__global__ void __launch_bounds__(kSingleThreads, 1)
    moe_single_kernel(const __grid_constant__ CUtensorMap tm1A, const __grid_constant__ CUtensorMap tm1B0,
                      const __grid_constant__ CUtensorMap tm1B1, const __grid_constant__ CUtensorMap tm2A,
                      const __grid_constant__ CUtensorMap tm2A1, const __grid_constant__ CUtensorMap tm2B0,
                      const GemmArgs a1, const GemmArgs a2) {
  static_assert(MODE2 == kStage2Pad || MODE2 == kStage2Comb, "second phase is a Stage2");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ctl = smem + kSingleRingBytes;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctl + 4);
  uint64_t* bars1 = reinterpret_cast<uint64_t*>(ctl + 8);
  uint64_t* bars2 = bars1 + kSingleBars1;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) *abort_flag = 0;
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  gemm_phase<kStage1, OutT, kQ16, 256, 1, 4, 5, kATma, 1, 1, 8>(&tm1A, &tm1A, &tm1B0, &tm1B1, a1, smem, bars1,
                                                                 tmem_slot, abort_flag, nullptr);
  // every role of the first phase has drained: the rings and TMEM are free for Stage2
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (!*abort_flag)
    gemm_phase<MODE2, OutT, kQ16, 256, 2, 3, 4, kATma, 1, 1, 8>(&tm2A, &tm2A1, &tm2B0, &tm2B0, a2, smem, bars2,
                                                                 tmem_slot, abort_flag, nullptr);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(*tmem_slot, kTmemCols);
  }
}

// ------------------------------------------------------------------ block groups
// Pairs the routing blocks of each expert: expert e owns blocks [gpo[e]/128, gpo[e+1]/128); they
// become ceil(n/gmax) groups of up to gmax consecutive blocks, in expert order. One CTA of 1024
// threads walks the experts in chunks of 1024 with a running base. At most max_groups groups are
// written (offsets that describe more blocks than the row space holds are cut off there). The
// kernel also clears zero[0..n_zero) (the single-kernel MoE's per-block Stage1 counts).
__global__ void __launch_bounds__(1024)
    build_groups_kernel(const int32_t* __restrict__ group_padded_offsets, int E, int gmax, int max_groups,
                        int32_t* __restrict__ groups, int32_t* __restrict__ ngroups_out,
                        uint32_t* __restrict__ zero, int n_zero) {
  __shared__ int s_warp[32];
  __shared__ int s_base;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  for (int i = tid; i < n_zero; i += blockDim.x) zero[i] = 0u;
  if (tid == 0) s_base = 0;
  __syncthreads();
  for (int e0 = 0; e0 < E; e0 += blockDim.x) {
    const int e = e0 + tid;
    int b0 = 0, nblk = 0;
    if (e < E) {
      b0 = group_padded_offsets[e] / kBM;
      nblk = group_padded_offsets[e + 1] / kBM - b0;
    }
    const int ng = (nblk + gmax - 1) / gmax;
    int incl = ng;
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
    const int base = s_base + incl - ng + (w > 0 ? s_warp[w - 1] : 0);
    for (int g = 0; g < ng && base + g < max_groups; ++g) {
      const int nb = min(gmax, nblk - g * gmax);
      groups[base + g] = (b0 + g * gmax) * 2 + (nb - 1);
    }
    __syncthreads();
    if (tid == 0) s_base += s_warp[31];
    __syncthreads();
  }
  if (tid == 0) *ngroups_out = min(s_base, max_groups);
}

}  // namespace moe
