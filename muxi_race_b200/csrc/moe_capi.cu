// moe_capi.cu — host side of the C ABI declared in include/moe_b200.h: argument checks, TMA
// descriptor encoding, workspace carving and the launch sequences of the three operator paths.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>

#include "../../include/moe_b200.h"
#include "ep_kernels.cuh"
#include "ep_p2p.cuh"
#include "gather_quant.cuh"
#include "moe_gemm.cuh"
#include "moe_gemm_pair.cuh"
#include "moe_gemm_tn.cuh"
#include "ordered_combine.cuh"
#include "route_align.cuh"
#include "router_topk.cuh"

namespace moe {

__device__ uint32_t g_status;  // device status word (kStatus* bits)

namespace {

thread_local std::string t_last_error;
thread_local void* const* t_prof_events = nullptr;
thread_local int t_prof_n = 0;

void prof_record(int i, cudaStream_t s) {
  if (t_prof_events && i < t_prof_n && t_prof_events[i]) cudaEventRecord(static_cast<cudaEvent_t>(t_prof_events[i]), s);
}

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

#define MOE_CUDA(call)                                                                        \
  do {                                                                                        \
    cudaError_t err_ = (call);                                                                \
    if (err_ != cudaSuccess)                                                                  \
      return fail(MOE_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(err_), __FILE__, __LINE__); \
  } while (0)

#define MOE_TRY(expr)          \
  do {                         \
    int rc_ = (expr);          \
    if (rc_ != MOE_OK) return rc_; \
  } while (0)

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  std::atomic<int> sms{0};
  std::atomic<uint32_t*> status{nullptr};
  std::atomic<uint64_t> attr_done[48] = {};  // bit per kernel whose smem attribute has been raised
};
DeviceInfo g_dev[kMaxDevices];

int current_device(int* dev) {
  MOE_CUDA(cudaGetDevice(dev));
  if (*dev < 0 || *dev >= kMaxDevices) return fail(MOE_ERR_UNSUPPORTED, "device ordinal %d out of range", *dev);
  return MOE_OK;
}

int device_sms(int dev, int* sms) {
  int v = g_dev[dev].sms.load(std::memory_order_relaxed);
  if (v == 0) {
    MOE_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
    g_dev[dev].sms.store(v, std::memory_order_relaxed);
  }
  *sms = v;
  return MOE_OK;
}

int device_status_ptr(int dev, uint32_t** p) {
  uint32_t* v = g_dev[dev].status.load(std::memory_order_acquire);
  if (v == nullptr) {
    MOE_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&v), g_status));
    g_dev[dev].status.store(v, std::memory_order_release);
  }
  *p = v;
  return MOE_OK;
}

template <typename K>
int raise_smem(int dev, int bit, K kernel, int bytes) {
  const uint64_t mask = uint64_t(1) << (bit & 63);
  std::atomic<uint64_t>& word = g_dev[dev].attr_done[bit >> 6];
  if (word.load(std::memory_order_acquire) & mask) return MOE_OK;
  MOE_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  word.fetch_or(mask, std::memory_order_acq_rel);
  return MOE_OK;
}

// ------------------------------------------------------------------ TMA descriptors
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// A grouped-GEMM tile configuration: accumulator columns per block (bn), blocks per work unit
// (gmax), A / B ring depths, CTAs per SM and k-blocks per weight box (kpb).
struct TileInfo {
  const char* name;
  int bn, gmax, ast, bst, cps, kpb;
  int pair;  // 1: CTA-pair kernel (cta_group::2), 256-row units, each CTA loads half the weights
  int epi;   // epilogue warps (4, or 8: two per TMEM lane quadrant, each half of the columns)
  int tn;    // 1: operand-swapped kernel (weights as M, an expert's tokens as N; fused path only)
  int kpa = 1;  // k-blocks per A box (one-block units on the TMA A path)
};

// Tiled map over a tensor of `rank` dimensions (dims[0] innermost, in elements; strides of dims
// 1..rank-1 in bytes), 128-byte swizzle (matches the kernels' shared-memory descriptors).
int encode_map(CUtensorMap* map, const void* base, int elt_bytes, int rank, const cuuint64_t* dims,
               const cuuint64_t* strides, const cuuint32_t* box, const char* what) {
  auto enc = get_encode();
  if (!enc) return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail(MOE_ERR_ALIGNMENT, "%s is not 16-byte aligned", what);
  for (int i = 0; i < rank; ++i)
    if (dims[i] == 0 || dims[i] > (cuuint64_t(1) << 31) - 1)
      return fail(MOE_ERR_INVALID_ARG, "%s has unsupported extent %llu in dimension %d", what,
                  (unsigned long long)dims[i], i);
  for (int i = 0; i + 1 < rank; ++i)
    if (strides[i] % 16 != 0 || strides[i] >= (cuuint64_t(1) << 40))
      return fail(MOE_ERR_ALIGNMENT, "%s stride %llu is not a multiple of 16 bytes below 2^40", what,
                  (unsigned long long)strides[i]);
  const CUtensorMapDataType dt = elt_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  static const CUtensorMapL2promotion promo = [] {
    const char* v = getenv("MOE_B200_L2_PROMO");  // experiments: none | 64 | 128 | 256 (default)
    if (v && strcmp(v, "none") == 0) return CU_TENSOR_MAP_L2_PROMOTION_NONE;
    if (v && strcmp(v, "64") == 0) return CU_TENSOR_MAP_L2_PROMOTION_L2_64B;
    if (v && strcmp(v, "128") == 0) return CU_TENSOR_MAP_L2_PROMOTION_L2_128B;
    return CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  }();
  CUresult r = enc(map, dt, rank, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed with %d", what, (int)r);
  return MOE_OK;
}

// Row-major [rows, cols] matrix, box = box_rows x (128 bytes).
int make_tmap(CUtensorMap* map, const void* base, int elt_bytes, int64_t rows, int64_t cols, int box_rows,
              const char* what) {
  if ((cols * elt_bytes) % 16 != 0) return fail(MOE_ERR_ALIGNMENT, "%s row pitch is not a multiple of 16 bytes", what);
  if (rows <= 0 || cols <= 0) return fail(MOE_ERR_INVALID_ARG, "%s has an empty extent", what);
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * elt_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kKBytes / elt_bytes), static_cast<cuuint32_t>(box_rows)};
  return encode_map(map, base, elt_bytes, 2, dims, strides, box, what);
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Tensor maps of one GEMM stage (see moe_gemm_kernel) and how the weight maps are laid out.
struct StageMaps {
  CUtensorMap a, a1, b0, b1;
  int b_split = 0;        // Stage1: gate and up rows as two maps (two boxes per k-block)
  int gu_swap = 0;        // Stage1 combined map based at the up rows
  int b1_row_offset = 0;  // Stage1 split: row offset of the up rows inside map b1
};

// A operand: one box per block group (gmax x 128 rows) and one per block; with kpa > 1 (one-block
// units) one 3-D box holds kpa consecutive 128-byte k-blocks of a block's rows (a k-block
// dimension of stride 128 bytes), which lands as kpa consecutive 128B-swizzled k-block tiles.
int make_a_maps(StageMaps* m, const void* base, int elt, int64_t rows, int64_t K, int gmax, const char* what,
                int kpa = 1) {
  if (kpa > 1) {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kKBytes / elt), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(K * elt / kKBytes)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(K * elt), static_cast<cuuint64_t>(kKBytes)};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(kKBytes / elt), static_cast<cuuint32_t>(kBM),
                               static_cast<cuuint32_t>(kpa)};
    MOE_TRY(encode_map(&m->a, base, elt, 3, dims, strides, box, what));
    m->a1 = m->a;
    return MOE_OK;
  }
  const int box = (gmax > 1 && rows >= gmax * kBM) ? gmax * kBM : kBM;  // fewer rows: no multi-block group
  MOE_TRY(make_tmap(&m->a, base, elt, rows, K, box, what));
  if (box != kBM) {
    MOE_TRY(make_tmap(&m->a1, base, elt, rows, K, kBM, what));
  } else {
    m->a1 = m->a;
  }
  return MOE_OK;
}

// Weights of a reduction length K stored as rows of K elements: one box of box_rows rows covers
// kpb consecutive 128-byte k-blocks (a k-block dimension of stride 128 bytes) when kpb > 1.
int make_w_map(CUtensorMap* map, const void* w, int elt, int64_t rows, int64_t K, int box_rows, int kpb,
               const char* what) {
  if (kpb == 1) return make_tmap(map, w, elt, rows, K, box_rows, what);
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kKBytes / elt), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(K * elt / kKBytes)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(K * elt), static_cast<cuuint64_t>(kKBytes)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kKBytes / elt), static_cast<cuuint32_t>(box_rows),
                             static_cast<cuuint32_t>(kpb)};
  return encode_map(map, w, elt, 3, dims, strides, box, what);
}

// Stage1 weights. Gate row r is at gate + r * K * elt and up row r at up + r * K * elt, for
// r < rows_gu. When the byte distance between the two is a multiple of 16 below 2^40, one map
// whose third dimension steps from the lower of the two to the other loads a tile's gate and up
// rows as one box (every address it forms is a row of one of the two tensors); otherwise two maps
// over split_gate / split_up (split_rows rows each, up rows at split_up_offset inside the second).
int make_stage1_weights(StageMaps* m, const void* gate, const void* up, int elt, int64_t rows_gu, int64_t K,
                        const TileInfo& t, const void* split_gate, const void* split_up, int64_t split_rows,
                        int split_up_offset, const char* what) {
  const uintptr_t g = reinterpret_cast<uintptr_t>(gate), u = reinterpret_cast<uintptr_t>(up);
  const uint64_t dist = g < u ? u - g : g - u;
  const int box_rows = t.bn / 2 < kMmaN ? t.bn / 2 : kMmaN;
  static const bool force_split = [] {
    const char* v = getenv("MOE_B200_B_SPLIT");  // experiments / tests: 1 = always two maps
    return v && strcmp(v, "1") == 0;
  }();
  if (!force_split && dist != 0 && dist % 16 == 0 && dist < (uint64_t(1) << 40) && (K * elt) % 16 == 0) {
    const void* lo = g < u ? gate : up;
    int rc;
    if (t.kpb == 1) {
      const cuuint64_t dims[3] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows_gu), 2};
      const cuuint64_t strides[2] = {static_cast<cuuint64_t>(K * elt), dist};
      const cuuint32_t box[3] = {static_cast<cuuint32_t>(kKBytes / elt), static_cast<cuuint32_t>(box_rows), 2};
      rc = encode_map(&m->b0, lo, elt, 3, dims, strides, box, what);
    } else {
      const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kKBytes / elt), static_cast<cuuint64_t>(rows_gu), 2,
                                  static_cast<cuuint64_t>(K * elt / kKBytes)};
      const cuuint64_t strides[3] = {static_cast<cuuint64_t>(K * elt), dist, static_cast<cuuint64_t>(kKBytes)};
      const cuuint32_t box[4] = {static_cast<cuuint32_t>(kKBytes / elt), static_cast<cuuint32_t>(box_rows), 2,
                                 static_cast<cuuint32_t>(t.kpb)};
      rc = encode_map(&m->b0, lo, elt, 4, dims, strides, box, what);
    }
    if (rc == MOE_OK) {
      m->b1 = m->b0;
      m->b_split = 0;
      m->gu_swap = u < g ? 1 : 0;
      return MOE_OK;
    }
  }
  MOE_TRY(make_tmap(&m->b0, split_gate, elt, split_rows, K, box_rows, what));
  MOE_TRY(make_tmap(&m->b1, split_up, elt, split_rows, K, box_rows, what));
  m->b_split = 1;
  m->gu_swap = 0;
  m->b1_row_offset = split_up_offset;
  return MOE_OK;
}

// ------------------------------------------------------------------ GEMM launch
// Tile configurations: accumulator columns per block (BN), blocks per work unit (GMAX), A / B
// ring depths, CTAs per SM and k-blocks per weight box (KPB). Names: <BN>[x<GMAX>]a<A>b<B>
// [c<CPS>][k<KPB>]. MOE_B200_TILE selects one by name for experiments (both stages),
// MOE_B200_TILE1 / MOE_B200_TILE2 one stage each.
enum TileCfg {
  kT256A4B5 = 0,
  kT256x2A3B4,
  kT512A2B3,
  kT256A2B2C2,
  kT256A6B4,
  kT256A6B2K2,
  kT128x2A3B4K2,
  kT128x2A4B3K2,
  kT128x2A3B8,
  kT256x2A3B2K2,
  kTP256A6B8,
  kTP256A7B7,
  kTP256A4B10,
  kT256A4B5E8,
  kT256x2A3B4E8,
  kTTN,
  kT128x2A4B6E8,
  kT256A3B4E8KA2,
  kT256A2B3E8KA4,
  kT256A3B2E8K2KA2,
  kT256A2B6E8,
  kT256A3B5E8,
  kT256X2A2B5E8,
  kT256A5B4E8,
  kT256A6B4E8,
  kT256X2A4B3E8,
  kNumTileCfg
};
constexpr TileInfo kTiles[kNumTileCfg] = {
    {"256a4b5", 256, 1, 4, 5, 1, 1, 0, 4},     {"256x2a3b4", 256, 2, 3, 4, 1, 1, 0, 4},
    {"512a2b3", 512, 1, 2, 3, 1, 1, 0, 4},     {"256a2b2c2", 256, 1, 2, 2, 2, 1, 0, 4},
    {"256a6b4", 256, 1, 6, 4, 1, 1, 0, 4},     {"256a6b2k2", 256, 1, 6, 2, 1, 2, 0, 4},
    {"128x2a3b4k2", 128, 2, 3, 4, 1, 2, 0, 4}, {"128x2a4b3k2", 128, 2, 4, 3, 1, 2, 0, 4},
    {"128x2a3b8", 128, 2, 3, 8, 1, 1, 0, 4},   {"256x2a3b2k2", 256, 2, 3, 2, 1, 2, 0, 4},
    {"p256a6b8", 256, 2, 6, 8, 1, 1, 1, 4},    {"p256a7b7", 256, 2, 7, 7, 1, 1, 1, 4},
    {"p256a4b10", 256, 2, 4, 10, 1, 1, 1, 4},  {"256a4b5e8", 256, 1, 4, 5, 1, 1, 0, 8},
    {"256x2a3b4e8", 256, 2, 3, 4, 1, 1, 0, 8}, {"tn", 256, 1, 6, 4, 1, 1, 0, 4, 1},
    {"128x2a4b6e8", 128, 2, 4, 6, 1, 1, 0, 8},
    {"256a3b4e8ka2", 256, 1, 3, 4, 1, 1, 0, 8, 0, 2}, {"256a2b3e8ka4", 256, 1, 2, 3, 1, 1, 0, 8, 0, 4},
    {"256a3b2e8k2ka2", 256, 1, 3, 2, 1, 2, 0, 8, 0, 2},
    {"256a2b6e8", 256, 1, 2, 6, 1, 1, 0, 8},   {"256a3b5e8", 256, 1, 3, 5, 1, 1, 0, 8},
    {"256x2a2b5e8", 256, 2, 2, 5, 1, 1, 0, 8}, {"256a5b4e8", 256, 1, 5, 4, 1, 1, 0, 8},
    {"256a6b4e8", 256, 1, 6, 4, 1, 1, 0, 8},   {"256x2a4b3e8", 256, 2, 4, 3, 1, 1, 0, 8},
};

// Defaults, measured on B200. Stage1: 256a4b5e8 (single CTA, 8 epilogue warps: the SiLU*up
// epilogue no longer holds up the next unit; cfg2 Stage1 0.52 vs 0.60-0.73 ms). Stage2, chosen per
// call from the average number of 128-row blocks per expert: from about 1.8 blocks per expert on,
// most blocks belong to two-block groups and the CTA-pair kernel p256a6b8 (one weight stream per
// two blocks, a third less shared-memory traffic per output) is fastest (cfg2 Stage2 0.31 vs
// 0.35 ms); below that, one-block groups would leave half of each pair idle (cfg3 at T = 128:
// 1.6 vs 1.1 ms) and 256x2a3b4e8 (single CTA, two-block groups sharing one weight stream, 8
// epilogue warps; cfg4 Stage2 0.83 vs 0.94 ms with 4) is used. With many blocks per expert the
// single-CTA tile wins again: an expert's several two-block groups read each weight tile at the
// same time on neighbouring SMs (expert-interleaved unit order), so the second and later reads
// hit L2 and the pair's shared weight stream saves nothing (cfg5, ~8.5 blocks per expert: Stage2
// 8.9-9.2 ms single-CTA against 9.8-10.1 ms for the pairs; cfg2, ~2.5: 0.342 against 0.318 ms
// for the pair). The pair is therefore chosen between 1.8 and 6 blocks per expert. MOE_B200_TILE /
// MOE_B200_TILE1 / MOE_B200_TILE2 or moe_set_tile override the choice with a configuration name.
TileCfg parse_tile(const char* v, TileCfg dflt) {
  if (v)
    for (int i = 0; i < kNumTileCfg; ++i)
      if (strcmp(v, kTiles[i].name) == 0) return static_cast<TileCfg>(i);
  return dflt;
}
constexpr TileCfg kDefaultTile1 = kT256A4B5E8, kDefaultTile2 = kT256x2A3B4E8, kDefaultPair = kTP256A6B8;
constexpr double kPairBlocksPerExpert = 1.8, kPairBlocksPerExpertMax = 6.0;
constexpr TileCfg kAuto = kNumTileCfg;
// Selected configuration per stage (kAuto = per-call choice): environment at first use,
// moe_set_tile afterwards.
std::atomic<int> g_tile_sel[2] = {{-1}, {-1}};
TileCfg tile_cfg(int stage) {
  std::atomic<int>& sel = g_tile_sel[stage == 1 ? 0 : 1];
  int v = sel.load(std::memory_order_acquire);
  if (v < 0) {
    const TileCfg env = parse_tile(getenv(stage == 1 ? "MOE_B200_TILE1" : "MOE_B200_TILE2"),
                                   parse_tile(getenv("MOE_B200_TILE"), kAuto));
    int expected = -1;
    sel.compare_exchange_strong(expected, static_cast<int>(env), std::memory_order_acq_rel);
    v = sel.load(std::memory_order_acquire);
  }
  return static_cast<TileCfg>(v);
}

// How Stage1's A operand is loaded (see AMode): MOE_B200_A_PATH = tma (a gather kernel stacks the
// token rows, TMA boxes read the stack) | lsu (cp.async gather in the GEMM) | gather (TMA
// tile::gather4 loads of the token rows in the GEMM, no stacked copy). Unset: kDefaultAPath.
enum APath : int { kAPathTma = 0, kAPathLsu = 1, kAPathGather = 2 };
constexpr int kDefaultAPath = kAPathTma;
int parse_a_path(const char* e) {
  if (e && strcmp(e, "lsu") == 0) return kAPathLsu;
  if (e && strcmp(e, "gather") == 0) return kAPathGather;
  if (e && strcmp(e, "tma") == 0) return kAPathTma;
  return -1;
}
// Selected A path: environment at first use, moe_set_a_path afterwards.
std::atomic<int> g_a_path{-1};
int a_path() {
  int v = g_a_path.load(std::memory_order_acquire);
  if (v < 0) {
    const int env = parse_a_path(getenv("MOE_B200_A_PATH"));
    int expected = -1;
    g_a_path.compare_exchange_strong(expected, env >= 0 ? env : kDefaultAPath, std::memory_order_acq_rel);
    v = g_a_path.load(std::memory_order_acquire);
  }
  return v;
}
bool a_path_lsu() { return a_path() == kAPathLsu; }
bool a_path_gather() { return a_path() == kAPathGather; }

// The configuration a stage runs with for reduction length K (elements of elt bytes), given the
// average number of 128-row blocks per expert: the selected one if any, else the per-call
// default. A weight box spanning KPB k-blocks needs whole k-blocks (K * elt a multiple of 128
// bytes) in multiples of KPB; BN = 128 is a Stage1 tile; the LSU A path (row table in shared
// memory) runs the single-CTA, 4-epilogue-warp, KPB = 1, BN >= 256 configurations. Anything else
// falls back to 256a4b5 / 256x2a3b4, which run on every path.
TileCfg usable_cfg(int stage, int64_t K, int elt, bool lsu, double blocks_per_expert) {
  const TileCfg safe = stage == 1 ? kT256A4B5 : kT256x2A3B4;
  TileCfg c = tile_cfg(stage);
  if (c == kAuto) {
    if (stage == 2 && !lsu && blocks_per_expert >= kPairBlocksPerExpert &&
        blocks_per_expert < kPairBlocksPerExpertMax)
      c = kDefaultPair;
    else
      c = stage == 1 ? kDefaultTile1 : kDefaultTile2;
  }
  const TileInfo& t = kTiles[c];
  if (t.kpb > 1 && ((K * elt) % kKBytes != 0 || ((K * elt) / kKBytes) % t.kpb != 0)) return safe;
  if (t.kpa > 1 && ((K * elt) % kKBytes != 0 || ((K * elt) / kKBytes) % t.kpa != 0)) return safe;
  if (t.bn == 128 && stage != 1 && c != kT128x2A4B6E8) return safe;  // 128-wide Stage2: this tile only
  if (lsu && (t.kpb > 1 || t.kpa > 1 || t.bn == 128 || t.pair || t.epi != 4)) return safe;
  if (t.tn && (lsu || (K * elt) % kKBytes != 0)) return safe;
  return c;
}
// Stage1 configurations built for the tile::gather4 A path (single CTA, one weight k-block per box)
bool gather_cfg(TileCfg c) { return c == kT256A4B5 || c == kT256A4B5E8 || c == kT256x2A3B4 || c == kT256x2A3B4E8; }
// Peer-memory EP gather: MOE_B200_EP_GATHER = dedup (default) selects
// gather_rows_peer_dedup_kernel (each token row read over NVLink once per rank, stored into all
// its local slots), route the per-route 16-byte load loop (one read per local route), bulk
// gather_rows_peer_bulk_kernel (bulk copies through shared memory), fused Stage1's gather warps
// (launch_stage1_gather_warps: no gather launch, the copies overlap the weight stream). Measured
// at 4096 tokens per rank: gather 0.17 vs 0.41 ms on 2 GPUs; on 8 GPUs the step 4.13 ms with
// dedup; fused on 2 GPUs: Stage1 grows by more than the gather it absorbs.
constexpr size_t kEpBulkMaxSmem = 220 * 1024;
enum EpGather : int { kEpGatherRoute = 0, kEpGatherBulk = 1, kEpGatherDedup = 2, kEpGatherFused = 3 };
static int ep_gather_mode() {
  static const int v = [] {
    const char* e = getenv("MOE_B200_EP_GATHER");
    if (e && strcmp(e, "bulk") == 0) return (int)kEpGatherBulk;
    if (e && strcmp(e, "route") == 0) return (int)kEpGatherRoute;
    if (e && strcmp(e, "fused") == 0) return (int)kEpGatherFused;
    return (int)kEpGatherDedup;
  }();
  return v;
}

// Unit order (see tile_unit): MOE_B200_UNIT_ORDER = expert (default: an expert's groups side by
// side per column tile) | group (group-major).
constexpr int kDefaultWeightsEvictFirst = 0;

int unit_order() {
  static const int v = [] {
    const char* e = getenv("MOE_B200_UNIT_ORDER");
    return (e && strcmp(e, "group") == 0) ? 0 : 1;
  }();
  return v;
}

// Bit of a kernel instantiation in the per-device "shared-memory attribute raised" mask: one
// range for moe_gemm_kernel (mode x element type x operand kind x configuration x A mode), one
// after it for the CTA-pair and operand-swapped kernels; the ranges must not overlap.
constexpr int kSmemKinds = 3 * 2 * 3;  // stage mode x 16-bit element type x operand kind
constexpr int kSmemBitsGemm = kSmemKinds * kNumTileCfg * 4;
constexpr int kSmemBitsOther = kSmemKinds * kNumTileCfg * 2;
static_assert(kSmemBitsGemm + kSmemBitsOther <= 64 * 48, "attr_done holds 48 words of bits");
constexpr int smem_bit_gemm(int mode, bool bf16, int q8, int tcfg, int amode) {
  return (((mode * 2 + (bf16 ? 1 : 0)) * 3 + q8) * kNumTileCfg + tcfg) * 4 + amode;
}
constexpr int smem_bit_other(int mode, bool bf16, int q8, int tcfg, int which) {
  return kSmemBitsGemm + (((mode * 2 + (bf16 ? 1 : 0)) * 3 + q8) * kNumTileCfg + tcfg) * 2 + which;
}

// L2 policy of the weight stream: MOE_B200_B_EVICT_FIRST = 0 (evict_normal in both stages), 1
// (evict_first in both), 2 (evict_first in Stage2 only); unset: kDefaultWeightsEvictFirst. Stage2
// reads each weight tile once (all blocks of an expert share one unit), while its combine adds
// every routed row into the token-major output; with evict_first the streamed weights leave L2
// first and the output rows stay. Stage1's weight tiles are read by the expert's neighbouring
// units, whose second reads hit L2. Read at each launch (a tuning switch: comparisons can flip it
// between calls of one process).
int weights_evict_first(int mode) {
  const char* e = getenv("MOE_B200_B_EVICT_FIRST");
  int v = kDefaultWeightsEvictFirst;
  if (e && (strcmp(e, "0") == 0 || strcmp(e, "1") == 0 || strcmp(e, "2") == 0)) v = e[0] - '0';
  return v == 1 || (v == 2 && mode != kStage1) ? 1 : 0;
}
// L2 policy of the Stage2 combine's adds into the token-major output: MOE_B200_OUT_EVICT_LAST =
// 0 (evict_normal) | 1 (evict_last: a token's rows stay in L2 between its top-k adds while the
// weights stream past); unset: kDefaultOutEvictLast. Read at each launch.
constexpr int kDefaultOutEvictLast = 0;
int out_evict_last() {
  const char* e = getenv("MOE_B200_OUT_EVICT_LAST");
  if (e && strcmp(e, "0") == 0) return 0;
  if (e && strcmp(e, "1") == 0) return 1;
  return kDefaultOutEvictLast;
}
// M = 64 MMAs for an expert's last block when it holds at most 64 valid rows (see half_block):
// MOE_B200_M64_TAIL = 0 | 1, unset: kDefaultM64Tail. Read at each launch.
constexpr int kDefaultM64Tail = 0;
int m64_tail() {
  const char* e = getenv("MOE_B200_M64_TAIL");
  if (e && strcmp(e, "0") == 0) return 0;
  if (e && strcmp(e, "1") == 0) return 1;
  return kDefaultM64Tail;
}
// Epilogue slot hand-back: MOE_B200_EPI_RELEASE = late hands the accumulator slot back after the
// epilogue's stores instead of right after its TMEM reads (comparison runs only; read at each
// launch).
int epilogue_late_release() {
  const char* e = getenv("MOE_B200_EPI_RELEASE");
  return e && strcmp(e, "late") == 0 ? 1 : 0;
}

// Single-kernel MoE (moe_single_kernel, Stage1 and Stage2 in one cooperative launch): mode 0 =
// two launches, 1 = the single kernel wherever it applies, 2 = automatic: where it applies and the
// call averages fewer than kPairBlocksPerExpert routing blocks per expert (the regime whose Stage2
// is the single-CTA two-block tile by choice). It applies where both stages run their default
// single-CTA tiles on the TMA A path (fp16/bf16 routes without the ordered combine or peer memory,
// no tile forced). Measured against the two launches on one B200, alternating in one process:
// cfg3 4.72 vs 4.78 ms, contest case 3 1.105 vs 1.121 ms, cfg3 at T = 128 3.44 vs 3.47 ms, but
// cfg5 (8.5 blocks per expert) 28.13 vs 27.88 ms. MOE_B200_SINGLE_KERNEL = 0 | 1 | 2 at first use,
// moe_set_single_kernel afterwards; unset: kDefaultSingleKernel.
constexpr int kDefaultSingleKernel = 2;
std::atomic<int> g_single_kernel{-1};
int single_kernel_mode() {
  int v = g_single_kernel.load(std::memory_order_acquire);
  if (v < 0) {
    const char* e = getenv("MOE_B200_SINGLE_KERNEL");
    const int env = e && (e[0] == '0' || e[0] == '1' || e[0] == '2') && e[1] == 0 ? e[0] - '0' : kDefaultSingleKernel;
    int expected = -1;
    g_single_kernel.compare_exchange_strong(expected, env, std::memory_order_acq_rel);
    v = g_single_kernel.load(std::memory_order_acquire);
  }
  return v;
}
// Whether a call that the single kernel covers runs it, given its average blocks per expert.
bool single_kernel(double blocks_per_expert) {
  const int mode = single_kernel_mode();
  return mode == 1 || (mode == 2 && blocks_per_expert < kPairBlocksPerExpert);
}
// The single kernel's shared-memory attribute bit: the operand-swapped kernel's range at a
// configuration that kernel never runs with (Stage2 modes); the Stage1 kernel with gather warps
// takes the Stage1 mode's bit there.
constexpr int smem_bit_single(int mode2, bool bf16) { return smem_bit_other(mode2, bf16, kQ16, kT256A4B5E8, 1); }
constexpr int smem_bit_gather_warps(bool bf16) { return smem_bit_other(kStage1, bf16, kQ16, kT256A4B5E8, 1); }

// Stage1 (tile 256a4b5e8) with 4 gather warps that copy the routed token rows from the peers'
// regions while the weights stream (expert parallelism over peer memory, MOE_B200_EP_GATHER =
// fused). Cooperative: every CTA's gather warps run, so every block the A producers wait for fills.
constexpr int kGatherWarps = 4;
template <typename OutT>
int launch_stage1_gather_warps(int dev, const StageMaps& m, const GemmArgs& args, int max_tiles, cudaStream_t stream) {
  auto kern = moe_gemm_kernel<kStage1, OutT, kQ16, 256, 1, 4, 5, kATma, 1, 1, 8, 1, kGatherWarps>;
  GemmArgs a = args;
  a.b_evict_first = weights_evict_first(kStage1);
  a.late_release = epilogue_late_release();
  a.m64_tail = m64_tail();
  a.unit_order = a.group_padded_offsets ? unit_order() : 0;
  a.b_split = m.b_split;
  a.gu_swap = m.gu_swap;
  if (m.b_split) a.b1_row_offset = m.b1_row_offset;
  constexpr int smem = Ring<256, 1, 4, 5>::kSmemBytes;
  MOE_TRY(raise_smem(dev, smem_bit_gather_warps(Elt<OutT>::kBF16), kern, smem));
  int sms = 0;
  MOE_TRY(device_sms(dev, &sms));
  const int grid = max_tiles < sms ? max_tiles : sms;
  if (grid <= 0) return MOE_OK;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(96 + 32 * 8 + 32 * kGatherWarps, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MOE_CUDA(cudaLaunchKernelEx(&cfg, kern, m.a, m.a1, m.b0, m.b1, a));
  return MOE_OK;
}

template <typename OutT, int MODE2>
int launch_single(int dev, const StageMaps& m1, const GemmArgs& a1, const StageMaps& m2, const GemmArgs& a2,
                  int max_tiles1, cudaStream_t stream) {
  auto kern = moe_single_kernel<OutT, MODE2>;
  GemmArgs x1 = a1, x2 = a2;
  for (GemmArgs* x : {&x1, &x2}) {
    x->out_evict_last = out_evict_last();
    x->late_release = epilogue_late_release();
    x->m64_tail = m64_tail();
    x->unit_order = x->group_padded_offsets ? unit_order() : 0;
  }
  x1.b_evict_first = weights_evict_first(kStage1);
  x2.b_evict_first = weights_evict_first(MODE2);
  x1.b_split = m1.b_split;
  x1.gu_swap = m1.gu_swap;
  if (m1.b_split) x1.b1_row_offset = m1.b1_row_offset;
  x2.b_split = 0;
  x2.gu_swap = 0;
  MOE_TRY(raise_smem(dev, smem_bit_single(MODE2, Elt<OutT>::kBF16), kern, kSingleSmemBytes));
  int sms = 0;
  MOE_TRY(device_sms(dev, &sms));
  const int grid = max_tiles1 < sms ? max_tiles1 : sms;
  if (grid <= 0) return MOE_OK;
  // cooperative: every CTA is resident at once (a Stage2 unit waits for other CTAs' Stage1 units)
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kSingleThreads, 1, 1);
  cfg.dynamicSmemBytes = kSingleSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MOE_CUDA(cudaLaunchKernelEx(&cfg, kern, m1.a, m1.b0, m1.b1, m2.a, m2.a1, m2.b0, x1, x2));
  return MOE_OK;
}
template <int MODE2>
int launch_single_rt(int dtype, int dev, const StageMaps& m1, const GemmArgs& a1, const StageMaps& m2,
                     const GemmArgs& a2, int max_tiles1, cudaStream_t stream) {
  if (dtype == MOE_F16) return launch_single<__half, MODE2>(dev, m1, a1, m2, a2, max_tiles1, stream);
  return launch_single<__nv_bfloat16, MODE2>(dev, m1, a1, m2, a2, max_tiles1, stream);
}

template <int MODE, typename OutT, int I8, int BN, int GMAX, int AST, int BST, int AMODE, int CPS, int KPB,
          int EPI = 4, int KPA = 1>
int launch_gemm(int dev, int tcfg, const StageMaps& m, const GemmArgs& args, int max_tiles, cudaStream_t stream) {
  auto kern = moe_gemm_kernel<MODE, OutT, I8, BN, GMAX, AST, BST, AMODE, CPS, KPB, EPI, KPA>;
  GemmArgs args_l = args;
  args_l.b_evict_first = weights_evict_first(MODE);
  args_l.out_evict_last = out_evict_last();
  args_l.late_release = epilogue_late_release();
  args_l.m64_tail = m64_tail();
  args_l.unit_order = args.group_padded_offsets ? unit_order() : 0;
  args_l.b_split = m.b_split;
  args_l.gu_swap = m.gu_swap;
  if (m.b_split) args_l.b1_row_offset = m.b1_row_offset;
  const int bit = smem_bit_gemm(MODE, Elt<OutT>::kBF16, I8, tcfg, AMODE);
  constexpr int smem = Ring<BN, GMAX, AST, BST, CPS, a_mode_lsu(AMODE), KPB, KPA>::kSmemBytes;
  MOE_TRY(raise_smem(dev, bit, kern, smem));
  int sms = 0;
  MOE_TRY(device_sms(dev, &sms));
  const int grid = max_tiles < sms * CPS ? max_tiles : sms * CPS;
  if (grid <= 0) return MOE_OK;
  kern<<<grid, 96 + 32 * EPI, smem, stream>>>(m.a, m.a1, m.b0, m.b1, args_l);
  MOE_CUDA(cudaGetLastError());
  return MOE_OK;
}

// CTA-pair kernel: clusters of two CTAs, one pair per two SMs (as many as can be resident).
template <int MODE, typename OutT, int I8, int AST, int BST, int EPI = 4>
int launch_pair(int dev, int tcfg, const StageMaps& m, const GemmArgs& args, int max_tiles, cudaStream_t stream) {
  auto kern = moe_gemm_pair_kernel<MODE, OutT, I8, AST, BST, EPI>;
  GemmArgs args_l = args;
  args_l.b_evict_first = weights_evict_first(MODE);
  args_l.out_evict_last = out_evict_last();
  args_l.late_release = epilogue_late_release();
  args_l.m64_tail = 0;  // the CTA-pair kernel's MMAs are M = 256
  args_l.unit_order = args.group_padded_offsets ? unit_order() : 0;
  args_l.b_split = 1;
  args_l.gu_swap = 0;
  args_l.b1_row_offset = m.b1_row_offset;
  const int bit = smem_bit_other(MODE, Elt<OutT>::kBF16, I8, tcfg, 0);
  constexpr int smem = PairRing<AST, BST>::kSmemBytes;
  MOE_TRY(raise_smem(dev, bit, kern, smem));
  static int max_pairs[kMaxDevices] = {};
  if (max_pairs[dev] == 0) {
    int sms = 0;
    MOE_TRY(device_sms(dev, &sms));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1), 1, 1);
    cfg.blockDim = dim3(96 + 32 * EPI, 1, 1);
    cfg.dynamicSmemBytes = smem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sms / 2;
    }
    max_pairs[dev] = n;
  }
  const int pairs = max_tiles < max_pairs[dev] ? max_tiles : max_pairs[dev];
  if (pairs <= 0) return MOE_OK;
  kern<<<2 * pairs, 96 + 32 * EPI, smem, stream>>>(m.a, m.b0, m.b1, args_l);
  MOE_CUDA(cudaGetLastError());
  return MOE_OK;
}

// Tensor maps of the operand-swapped kernel: the weights and the token rows in boxes of 128 /
// 64 / 32 / 16 rows.
struct TnMaps {
  CUtensorMap w, x128, x64, x32, x16;
};

int make_tn_x_maps(TnMaps* m, const void* rows_base, int elt, int64_t rows, int64_t K, const char* what) {
  MOE_TRY(make_tmap(&m->x128, rows_base, elt, rows, K, 128, what));
  MOE_TRY(make_tmap(&m->x64, rows_base, elt, rows, K, 64, what));
  MOE_TRY(make_tmap(&m->x32, rows_base, elt, rows, K, 32, what));
  MOE_TRY(make_tmap(&m->x16, rows_base, elt, rows, K, 16, what));
  return MOE_OK;
}

// Stage1 weights of the fused path: 5-D map {k-block elements, 8 rows, gate/up, 8-row groups,
// k-blocks} over w_gate_up [E, 2I, H] (gate rows at e*2I + f, up rows I further), box
// {64, 8, 2, 8, 1}: 64 gate and 64 up rows interleaved by 8-row atoms.
int make_tn_w13_map(CUtensorMap* map, const void* w13, int elt, int64_t E, int64_t H, int64_t I) {
  if (I % 8 != 0 || (H * elt) % kKBytes != 0)
    return fail(MOE_ERR_UNSUPPORTED, "operand-swapped Stage1 needs I a multiple of 8 and whole 128-byte k-blocks");
  const cuuint64_t dims[5] = {static_cast<cuuint64_t>(kKBytes / elt), 8, 2,
                              static_cast<cuuint64_t>((2 * E * I - I) / 8), static_cast<cuuint64_t>(H * elt / kKBytes)};
  const cuuint64_t strides[4] = {static_cast<cuuint64_t>(H * elt), static_cast<cuuint64_t>(I * H * elt),
                                 static_cast<cuuint64_t>(8 * H * elt), static_cast<cuuint64_t>(kKBytes)};
  const cuuint32_t box[5] = {static_cast<cuuint32_t>(kKBytes / elt), 8, 2, 8, 1};
  return encode_map(map, w13, elt, 5, dims, strides, box, "w_gate_up (operand-swapped)");
}

template <int MODE, typename OutT, int Q8>
int launch_tn(int dev, int tcfg, const TnMaps& m, const TnArgs& args, int max_units, cudaStream_t stream) {
  constexpr int AST = 6, BST = 4;
  auto kern = moe_gemm_tn_kernel<MODE, OutT, AST, BST, Q8>;
  const int bit = smem_bit_other(MODE, Elt<OutT>::kBF16, Q8, tcfg, 1);
  constexpr int smem = TnRing<AST, BST>::kSmemBytes;
  MOE_TRY(raise_smem(dev, bit, kern, smem));
  int sms = 0;
  MOE_TRY(device_sms(dev, &sms));
  const int grid = max_units < sms ? max_units : sms;
  if (grid <= 0) return MOE_OK;
  kern<<<grid, kThreads, smem, stream>>>(m.w, m.x128, m.x64, m.x32, m.x16, args);
  MOE_CUDA(cudaGetLastError());
  return MOE_OK;
}

template <int MODE, int Q8 = kQ16>
int launch_tn_rt(int dtype, int dev, int tcfg, const TnMaps& m, const TnArgs& args, int max_units, cudaStream_t s) {
  return dtype == MOE_F16 ? launch_tn<MODE, __half, Q8>(dev, tcfg, m, args, max_units, s)
                          : launch_tn<MODE, __nv_bfloat16, Q8>(dev, tcfg, m, args, max_units, s);
}

// One grouped GEMM stage with the chosen tile configuration.
// I8: operand kind (kQ16, kQI8, kQF8); the fp8 kind is built for the default tiles and the TMA A
// path only.
template <int MODE, typename OutT, int I8, int AMODE>
int launch_stage(TileCfg c, int dev, const StageMaps& m, const GemmArgs& args, int max_tiles, cudaStream_t stream) {
  constexpr bool kTma = AMODE == kATma;
  constexpr bool kS1 = MODE == kStage1;
  if constexpr (I8 == kQF8) {
    if constexpr (kTma) {
      switch (c) {
        case kT256A4B5:
          return launch_gemm<MODE, OutT, I8, 256, 1, 4, 5, AMODE, 1, 1>(dev, c, m, args, max_tiles, stream);
        case kT256x2A3B4:
          return launch_gemm<MODE, OutT, I8, 256, 2, 3, 4, AMODE, 1, 1>(dev, c, m, args, max_tiles, stream);
        case kT256A4B5E8:
          return launch_gemm<MODE, OutT, I8, 256, 1, 4, 5, AMODE, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
        case kT256x2A3B4E8:
          return launch_gemm<MODE, OutT, I8, 256, 2, 3, 4, AMODE, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
        case kTP256A6B8:
          return launch_pair<MODE, OutT, I8, 6, 8>(dev, c, m, args, max_tiles, stream);
        default:
          break;
      }
    }
    return fail(MOE_ERR_UNSUPPORTED, "tile configuration %s is not built for fp8 operands", kTiles[c].name);
  } else {
    switch (c) {
      case kT256A4B5:
        return launch_gemm<MODE, OutT, I8, 256, 1, 4, 5, AMODE, 1, 1>(dev, c, m, args, max_tiles, stream);
      case kT256x2A3B4:  // the LSU A path's row table does not fit next to this ring: 2-deep A there
        if constexpr (kTma)
          return launch_gemm<MODE, OutT, I8, 256, 2, 3, 4, AMODE, 1, 1>(dev, c, m, args, max_tiles, stream);
        else
          return launch_gemm<MODE, OutT, I8, 256, 2, 2, 4, AMODE, 1, 1>(dev, c, m, args, max_tiles, stream);
      case kT512A2B3:
        return launch_gemm<MODE, OutT, I8, 512, 1, 2, 3, AMODE, 1, 1>(dev, c, m, args, max_tiles, stream);
      case kT256A2B2C2:
        return launch_gemm<MODE, OutT, I8, 256, 1, 2, 2, AMODE, 2, 1>(dev, c, m, args, max_tiles, stream);
      case kT256A6B4:
        return launch_gemm<MODE, OutT, I8, 256, 1, 6, 4, AMODE, 1, 1>(dev, c, m, args, max_tiles, stream);
      case kT256A6B2K2:
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 1, 6, 2, AMODE, 1, 2>(dev, c, m, args, max_tiles, stream);
        break;
      case kT128x2A3B4K2:
        if constexpr (kTma && kS1)
          return launch_gemm<MODE, OutT, I8, 128, 2, 3, 4, AMODE, 1, 2>(dev, c, m, args, max_tiles, stream);
        break;
      case kT128x2A4B3K2:
        if constexpr (kTma && kS1)
          return launch_gemm<MODE, OutT, I8, 128, 2, 4, 3, AMODE, 1, 2>(dev, c, m, args, max_tiles, stream);
        break;
      case kT128x2A3B8:
        if constexpr (kTma && kS1)
          return launch_gemm<MODE, OutT, I8, 128, 2, 3, 8, AMODE, 1, 1>(dev, c, m, args, max_tiles, stream);
        break;
      case kT256x2A3B2K2:
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 2, 3, 2, AMODE, 1, 2>(dev, c, m, args, max_tiles, stream);
        break;
      case kTP256A6B8:
        if constexpr (kTma) return launch_pair<MODE, OutT, I8, 6, 8>(dev, c, m, args, max_tiles, stream);
        break;
      case kTP256A7B7:
        if constexpr (kTma) return launch_pair<MODE, OutT, I8, 7, 7>(dev, c, m, args, max_tiles, stream);
        break;
      case kTP256A4B10:
        if constexpr (kTma) return launch_pair<MODE, OutT, I8, 4, 10>(dev, c, m, args, max_tiles, stream);
        break;
      case kT256A4B5E8:
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 1, 4, 5, AMODE, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
        break;
      case kT256x2A3B4E8:
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 2, 3, 4, AMODE, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
        break;
      case kT128x2A4B6E8:  // two-block groups, 128 columns per block: two units' accumulators in TMEM
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 128, 2, 4, 6, AMODE, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
        break;
      case kT256A2B6E8:  // deeper weight rings, shallower token-row rings
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 1, 2, 6, AMODE, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
        break;
      case kT256A3B5E8:
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 1, 3, 5, AMODE, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
        break;
      case kT256X2A2B5E8:
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 2, 2, 5, AMODE, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
        break;
      case kT256A5B4E8:  // deeper token-row rings
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 1, 5, 4, AMODE, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
        break;
      case kT256A6B4E8:
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 1, 6, 4, AMODE, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
        break;
      case kT256X2A4B3E8:
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 2, 4, 3, AMODE, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
        break;
      case kT256A3B4E8KA2:  // A boxes of 2 k-blocks: fewer, larger TMA loads per unit
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 1, 3, 4, AMODE, 1, 1, 8, 2>(dev, c, m, args, max_tiles, stream);
        break;
      case kT256A2B3E8KA4:
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 1, 2, 3, AMODE, 1, 1, 8, 4>(dev, c, m, args, max_tiles, stream);
        break;
      case kT256A3B2E8K2KA2:
        if constexpr (kTma) return launch_gemm<MODE, OutT, I8, 256, 1, 3, 2, AMODE, 1, 2, 8, 2>(dev, c, m, args, max_tiles, stream);
        break;

      default:
        break;
    }
  }
  return fail(MOE_ERR_UNSUPPORTED, "tile configuration %s is not available for this stage", kTiles[c].name);
}

// Stage1 with the tile::gather4 A path (configurations of gather_cfg).
template <typename OutT, int I8>
int launch_stage1_gather(TileCfg c, int dev, const StageMaps& m, const GemmArgs& args, int max_tiles,
                         cudaStream_t stream) {
  switch (c) {
    case kT256A4B5:
      return launch_gemm<kStage1, OutT, I8, 256, 1, 4, 5, kATmaGather, 1, 1>(dev, c, m, args, max_tiles, stream);
    case kT256A4B5E8:
      return launch_gemm<kStage1, OutT, I8, 256, 1, 4, 5, kATmaGather, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
    case kT256x2A3B4:
      return launch_gemm<kStage1, OutT, I8, 256, 2, 3, 4, kATmaGather, 1, 1>(dev, c, m, args, max_tiles, stream);
    case kT256x2A3B4E8:
      return launch_gemm<kStage1, OutT, I8, 256, 2, 3, 4, kATmaGather, 1, 1, 8>(dev, c, m, args, max_tiles, stream);
    default:
      return fail(MOE_ERR_UNSUPPORTED, "tile configuration %s is not built for the gather4 A path", kTiles[c].name);
  }
}
template <int I8>
int launch_stage1_gather_rt(int dtype, TileCfg c, int dev, const StageMaps& m, const GemmArgs& args, int max_tiles,
                            cudaStream_t stream) {
  return dtype == MOE_F16 ? launch_stage1_gather<__half, I8>(c, dev, m, args, max_tiles, stream)
                          : launch_stage1_gather<__nv_bfloat16, I8>(c, dev, m, args, max_tiles, stream);
}

// Stage dispatch over the runtime element type and A path.
template <int MODE, int I8, int AMODE_LSU>
int launch_stage_rt(int dtype, bool lsu, TileCfg c, int dev, const StageMaps& m, const GemmArgs& args, int max_tiles,
                    cudaStream_t stream) {
  if (dtype == MOE_F16)
    return lsu ? launch_stage<MODE, __half, I8, AMODE_LSU>(c, dev, m, args, max_tiles, stream)
               : launch_stage<MODE, __half, I8, kATma>(c, dev, m, args, max_tiles, stream);
  return lsu ? launch_stage<MODE, __nv_bfloat16, I8, AMODE_LSU>(c, dev, m, args, max_tiles, stream)
             : launch_stage<MODE, __nv_bfloat16, I8, kATma>(c, dev, m, args, max_tiles, stream);
}

// ------------------------------------------------------------------ align
int align_chunk(int64_t R) {
  int64_t c = (R + 255) / 256;
  c = (c + 31) / 32 * 32;
  if (c < 256) c = 256;
  if (c > 4096) c = 4096;
  return static_cast<int>(c);
}
int64_t align_chunks(int64_t R) { return R <= 0 ? 0 : (R + align_chunk(R) - 1) / align_chunk(R); }

// counted: `counts` already holds the per-chunk histogram (built by the router kernel).
int launch_align(const void* ids, int ids_dtype, int64_t R, int64_t E, int64_t bm, int32_t* gs, int32_t* go,
                 int32_t* gpo, int32_t* gidx, int32_t* sorted, int32_t* route_slot, int32_t* meta, int* counts,
                 cudaStream_t stream, bool counted = false) {
  const int chunk = align_chunk(R);
  const int n_chunks = static_cast<int>(align_chunks(R));
  const int grid = (n_chunks + kAlignWarps - 1) / kAlignWarps;
  const size_t smem = sizeof(int) * kAlignWarps * E;
  if (n_chunks > 0 && !counted) {
    if (ids_dtype == MOE_I32)
      align_count_kernel<int32_t><<<grid, kAlignWarps * 32, smem, stream>>>(
          static_cast<const int32_t*>(ids), (int)R, (int)E, chunk, n_chunks, counts);
    else
      align_count_kernel<int64_t><<<grid, kAlignWarps * 32, smem, stream>>>(
          static_cast<const int64_t*>(ids), (int)R, (int)E, chunk, n_chunks, counts);
    MOE_CUDA(cudaGetLastError());
  }
  align_scan_kernel<<<1, 1024, 0, stream>>>(counts, n_chunks, (int)E, (int)bm, (int)R, gs, go, gpo, gidx, sorted, meta);
  MOE_CUDA(cudaGetLastError());
  if (n_chunks > 0) {
    if (ids_dtype == MOE_I32)
      align_scatter_kernel<int32_t><<<grid, kAlignWarps * 32, smem, stream>>>(
          static_cast<const int32_t*>(ids), (int)R, (int)E, chunk, n_chunks, counts, gpo, sorted, route_slot);
    else
      align_scatter_kernel<int64_t><<<grid, kAlignWarps * 32, smem, stream>>>(
          static_cast<const int64_t*>(ids), (int)R, (int)E, chunk, n_chunks, counts, gpo, sorted, route_slot);
    MOE_CUDA(cudaGetLastError());
  }
  return MOE_OK;
}

// Workspace carving for the token-major paths.
struct FusedLayout {
  size_t counts, gs, go, gpo, meta, gidx, groups, done, tn, sorted, slot, xs, xscale, u, uq, uscale, amax, y, raw,
      total;
  int64_t P_max, nblk_max;
};

// ordered: the padded Stage2 rows y [P_max, H] and raw-order weights [R] of the ordered combine.
FusedLayout fused_layout(int64_t T, int64_t topk, int64_t E, int64_t H, int64_t I, bool int8, bool lsu,
                         bool ordered = false) {
  FusedLayout L{};
  const int64_t R = T * topk;
  L.P_max = moe_max_padded_rows(R, E, kBM);
  L.nblk_max = L.P_max / kBM;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = round_up(off + bytes, 256);
    return o;
  };
  L.counts = take(sizeof(int) * (size_t)align_chunks(R) * E);
  L.gs = take(sizeof(int) * E);
  L.go = take(sizeof(int) * (E + 1));
  L.gpo = take(sizeof(int) * (E + 1));
  L.meta = take(sizeof(int) * 4);
  L.gidx = take(sizeof(int) * (size_t)L.nblk_max);
  L.groups = take(sizeof(int) * (size_t)(L.nblk_max + 1));  // block groups + their count
  // single kernel: Stage1 counts per block; fused peer gather: rows per block, then token claims
  L.done = take(sizeof(uint32_t) * (size_t)(L.nblk_max + T));
  L.tn = take(sizeof(int) * (size_t)(2 * L.nblk_max + 1));   // operand-swapped kernel: entries + count
  L.sorted = take(sizeof(int) * (size_t)L.P_max);
  L.slot = take(sizeof(int) * (size_t)R);
  // token rows: stacked per expert (TMA A path) or read in place (LSU gather; int8 quantised
  // per token first)
  const size_t a_rows = lsu ? (size_t)T : (size_t)L.P_max;
  L.xs = take(lsu ? (int8 ? a_rows * H : 0) : (int8 ? 1 : 2) * a_rows * H);
  L.xscale = take(int8 ? sizeof(float) * a_rows : 0);
  L.u = take(2 * (size_t)L.P_max * I);
  L.uq = take(int8 ? (size_t)L.P_max * I : 0);
  L.uscale = take(int8 ? sizeof(float) * (size_t)L.P_max : 0);
  L.amax = take(int8 ? sizeof(float) * (size_t)L.P_max : 0);
  L.y = take(ordered ? 2 * (size_t)L.P_max * H : 0);
  L.raw = take(ordered ? sizeof(float) * (size_t)R : 0);
  L.total = off;
  return L;
}

int check_common(int64_t H, int64_t I, int64_t E, int dtype, int mult) {
  if (dtype != MOE_F16 && dtype != MOE_BF16) return fail(MOE_ERR_INVALID_ARG, "dtype must be MOE_F16 or MOE_BF16");
  if (H <= 0 || I <= 0 || E <= 0) return fail(MOE_ERR_INVALID_ARG, "hidden, intermediate and experts must be > 0");
  if (H % mult != 0 || I % mult != 0)
    return fail(MOE_ERR_INVALID_ARG, "hidden (%lld) and intermediate (%lld) must be multiples of %d", (long long)H,
                (long long)I, mult);
  if (H > (1 << 30) || I > (1 << 30)) return fail(MOE_ERR_INVALID_ARG, "hidden/intermediate too large");
  return MOE_OK;
}

// ------------------------------------------------------------------ router
template <typename LogitT>
int launch_router_t(const LogitT* logits, int64_t T, int64_t E, int64_t topk, int renorm, int32_t* ids, float* w,
                    int* counts, int chunk, int n_chunks, int sms, cudaStream_t s) {
  const int64_t want = (T + kRouterWarps - 1) / kRouterWarps;
  const int grid = static_cast<int>(want < (int64_t)sms * 16 ? want : (int64_t)sms * 16);
  const int threads = kRouterWarps * 32;
#define MOE_ROUTER_CASE(V)                                                                                      \
  if (E <= 32 * (V)) {                                                                                          \
    router_topk_kernel<LogitT, V><<<grid, threads, 0, s>>>(logits, (int)T, (int)E, (int)topk, renorm, ids, w, \
                                                          counts, chunk, n_chunks);                           \
    MOE_CUDA(cudaGetLastError());                                                                               \
    return MOE_OK;                                                                                              \
  }
  MOE_ROUTER_CASE(1)
  MOE_ROUTER_CASE(2)
  MOE_ROUTER_CASE(4)
  MOE_ROUTER_CASE(8)
  MOE_ROUTER_CASE(16)
  MOE_ROUTER_CASE(32)
#undef MOE_ROUTER_CASE
  return fail(MOE_ERR_INVALID_ARG, "num_experts must be <= %d", 32 * 32);
}

int check_router(const void* logits, int logits_dtype, int64_t T, int64_t E, int64_t topk, const int32_t* ids,
                        const float* w) {
  if (logits_dtype != MOE_F32 && logits_dtype != MOE_F16 && logits_dtype != MOE_BF16)
    return fail(MOE_ERR_INVALID_ARG, "router logits must be fp32, fp16 or bf16");
  if (E < 1 || E > kAlignMaxExperts) return fail(MOE_ERR_INVALID_ARG, "num_experts must be in [1, %d]", kAlignMaxExperts);
  if (topk < 1 || topk > kRouterMaxTopk || topk > E)
    return fail(MOE_ERR_INVALID_ARG, "topk must be in [1, min(num_experts, %d)]", kRouterMaxTopk);
  if (T < 0 || T * topk > (int64_t(1) << 31) - 1) return fail(MOE_ERR_INVALID_ARG, "bad token count");
  if (T > 0 && (!logits || !ids || !w)) return fail(MOE_ERR_INVALID_ARG, "null tensor argument");
  return MOE_OK;
}

// Runs the router on `s`; with `counts` (zeroed here) it also builds the alignment histogram for
// R = T * topk routes.
int launch_router(const void* logits, int logits_dtype, int64_t T, int64_t E, int64_t topk, int renorm,
                         int32_t* ids, float* w, int* counts, cudaStream_t s) {
  int dev, sms;
  MOE_TRY(current_device(&dev));
  MOE_TRY(device_sms(dev, &sms));
  const int64_t R = T * topk;
  const int chunk = align_chunk(R);
  const int n_chunks = static_cast<int>(align_chunks(R));
  if (counts) MOE_CUDA(cudaMemsetAsync(counts, 0, sizeof(int) * (size_t)n_chunks * (size_t)E, s));
  renorm = renorm ? 1 : 0;
  if (logits_dtype == MOE_F32)
    return launch_router_t(static_cast<const float*>(logits), T, E, topk, renorm, ids, w, counts, chunk, n_chunks, sms,
                           s);
  if (logits_dtype == MOE_F16)
    return launch_router_t(static_cast<const __half*>(logits), T, E, topk, renorm, ids, w, counts, chunk, n_chunks,
                           sms, s);
  return launch_router_t(static_cast<const __nv_bfloat16*>(logits), T, E, topk, renorm, ids, w, counts, chunk,
                         n_chunks, sms, s);
}

template <typename LogitT>
int launch_router_grouped_t(const LogitT* logits, const float* bias, int64_t T, int64_t E, int64_t n_group,
                            int64_t topk_group, int64_t topk, int renorm, float scale, int32_t* ids, float* w, int sms,
                            cudaStream_t s) {
  const int64_t want = (T + kRouterWarps - 1) / kRouterWarps;
  const int grid = static_cast<int>(want < (int64_t)sms * 16 ? want : (int64_t)sms * 16);
  const int threads = kRouterWarps * 32;
  const size_t smem = sizeof(float) * kRouterWarps * static_cast<size_t>(E);
#define MOE_ROUTER_G_CASE(V)                                                                                  \
  if (E <= 32 * (V)) {                                                                                        \
    router_grouped_kernel<LogitT, V><<<grid, threads, smem, s>>>(logits, bias, (int)T, (int)E, (int)n_group,  \
                                                                 (int)topk_group, (int)topk, renorm, scale,   \
                                                                 ids, w);                                     \
    MOE_CUDA(cudaGetLastError());                                                                             \
    return MOE_OK;                                                                                            \
  }
  MOE_ROUTER_G_CASE(1)
  MOE_ROUTER_G_CASE(2)
  MOE_ROUTER_G_CASE(4)
  MOE_ROUTER_G_CASE(8)
  MOE_ROUTER_G_CASE(16)
  MOE_ROUTER_G_CASE(32)
#undef MOE_ROUTER_G_CASE
  return fail(MOE_ERR_INVALID_ARG, "num_experts must be <= %d", 32 * 32);
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" {

const char* moe_version(void) { return "muxi_race_b200 0.1.0 (sm_100a)"; }

const char* moe_last_error(void) { return t_last_error.c_str(); }

int moe_set_tile(int stage, const char* name) {
  t_last_error.clear();
  if (stage < 0 || stage > 2) return fail(MOE_ERR_INVALID_ARG, "stage must be 0, 1 or 2");
  TileCfg c = kAuto;
  if (name != nullptr && strcmp(name, "auto") != 0) {
    c = parse_tile(name, kAuto);
    if (c == kAuto) return fail(MOE_ERR_INVALID_ARG, "unknown tile configuration '%s'", name);
  }
  for (int st = 1; st <= 2; ++st)
    if (stage == 0 || stage == st) g_tile_sel[st - 1].store(static_cast<int>(c), std::memory_order_release);
  return MOE_OK;
}

int moe_set_single_kernel(int mode) {
  t_last_error.clear();
  if (mode < 0 || mode > 2) return fail(MOE_ERR_INVALID_ARG, "moe_set_single_kernel takes 0, 1 or 2");
  g_single_kernel.store(mode, std::memory_order_release);
  return MOE_OK;
}

int moe_set_a_path(const char* name) {
  t_last_error.clear();
  const int v = name == nullptr || strcmp(name, "auto") == 0 ? kDefaultAPath : parse_a_path(name);
  if (v < 0) return fail(MOE_ERR_INVALID_ARG, "unknown A path '%s' (tma, gather, lsu)", name);
  g_a_path.store(v, std::memory_order_release);
  return MOE_OK;
}

int moe_set_profile_events(void* const* events, int n) {
  t_prof_events = n > 0 ? events : nullptr;
  t_prof_n = n > 0 ? n : 0;
  return MOE_OK;
}

int moe_device_status(void* stream, int clear, uint32_t* status_out) {
  int dev;
  MOE_TRY(current_device(&dev));
  uint32_t* p;
  MOE_TRY(device_status_ptr(dev, &p));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  MOE_CUDA(cudaMemcpyAsync(&v, p, sizeof(v), cudaMemcpyDeviceToHost, s));
  MOE_CUDA(cudaStreamSynchronize(s));
  if (clear) {
    MOE_CUDA(cudaMemsetAsync(p, 0, sizeof(uint32_t), s));
    MOE_CUDA(cudaStreamSynchronize(s));
  }
  if (status_out) *status_out = v;
  return MOE_OK;
}

// ---------------------------------------------------------------------------- run_kernel
// Workspace: U [P, I] (the reference's cached up_logits) + block groups [P/128] + group count +
// the single kernel's per-block Stage1 counts [P/128].
static size_t run_kernel_u_bytes(int64_t P, int64_t I) { return round_up(static_cast<size_t>(P) * I * 2, 256); }
static size_t run_kernel_groups_bytes(int64_t P) {
  return round_up(sizeof(int32_t) * static_cast<size_t>(P / kBM + 1), 256);
}

size_t moe_run_kernel_workspace_bytes(int64_t P, int64_t I, int dtype) {
  (void)dtype;
  if (P <= 0 || I <= 0) return 0;
  return run_kernel_u_bytes(P, I) + run_kernel_groups_bytes(P) +
         round_up(sizeof(uint32_t) * static_cast<size_t>(P / kBM), 256);
}

int moe_run_kernel(const void* x, const void* gate_w, const void* up_w, const void* down_w, const void* routed,
                   int routed_dtype, const int32_t* gs, const int32_t* go, const int32_t* gpo, const int32_t* gidx,
                   void* out, int64_t P, int64_t H, int64_t I, int64_t E, int64_t R, int64_t nblk, int dtype,
                   void* workspace, size_t workspace_bytes, void* stream) {
  t_last_error.clear();
  MOE_TRY(check_common(H, I, E, dtype, 8));
  if (P < 0 || R < 0 || nblk < 0) return fail(MOE_ERR_INVALID_ARG, "negative size");
  if (P != nblk * kBM)
    return fail(MOE_ERR_INVALID_ARG, "total_padded_tokens (%lld) != 128 * num_blocks_m (%lld)", (long long)P,
                (long long)nblk);
  if (routed_dtype != MOE_F32 && routed_dtype != MOE_F16)
    return fail(MOE_ERR_INVALID_ARG, "routed_expert_weights must be fp32 or fp16");
  if (P > (int64_t(1) << 31) - 1 || R > (int64_t(1) << 31) - 1) return fail(MOE_ERR_INVALID_ARG, "too many rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (P == 0) return MOE_OK;  // SUB/submission.py:2117-2120
  if (!out || !aligned16(out)) return fail(MOE_ERR_ALIGNMENT, "out must be a 16-byte aligned device pointer");
  if (R == 0) {  // SUB/submission.py:2130-2153: no valid rows, Stage2 zero-fills the padded output
    MOE_CUDA(cudaMemsetAsync(out, 0, static_cast<size_t>(P) * H * 2, s));
    return MOE_OK;
  }
  if (!x || !gate_w || !up_w || !down_w || !routed || !gs || !go || !gpo || !gidx)
    return fail(MOE_ERR_INVALID_ARG, "null tensor argument");
  if (!workspace || workspace_bytes < moe_run_kernel_workspace_bytes(P, I, dtype))
    return fail(MOE_ERR_WORKSPACE, "workspace must hold %zu bytes", moe_run_kernel_workspace_bytes(P, I, dtype));
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return fail(MOE_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  if (E * I > (int64_t(1) << 31) - 1 || E * H > (int64_t(1) << 31) - 1)
    return fail(MOE_ERR_INVALID_ARG, "experts x rows exceeds the TMA coordinate range");
  int dev;
  MOE_TRY(current_device(&dev));
  uint32_t* status;
  MOE_TRY(device_status_ptr(dev, &status));
  void* U = workspace;
  int32_t* groups = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + run_kernel_u_bytes(P, I));
  int32_t* ngroups = groups + nblk;
  uint32_t* done = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + run_kernel_u_bytes(P, I) +
                                               run_kernel_groups_bytes(P));
  const bool lsu = a_path_lsu();
  const double bpe = static_cast<double>(nblk) / static_cast<double>(E);  // blocks per expert
  TileCfg tc1 = usable_cfg(1, H, 2, lsu, bpe), tc2 = usable_cfg(2, I, 2, lsu, bpe);
  if (kTiles[tc1].tn) tc1 = kT256A4B5;  // the operand-swapped kernel runs on the fused path only
  if (kTiles[tc2].tn) tc2 = kT256x2A3B4;
  // single-kernel MoE: both stages in one launch, on their default single-CTA tiles
  const bool single = single_kernel(bpe) && !lsu && tile_cfg(1) == kAuto && tile_cfg(2) == kAuto;
  if (single) {
    tc1 = kDefaultTile1;
    tc2 = kDefaultTile2;
  }
  const TileInfo &t1 = kTiles[tc1], &t2 = kTiles[tc2];
  const int bn1 = t1.bn, gmax1 = t1.gmax, bn2 = t2.bn, gmax2 = t2.gmax;

  StageMaps m1, m2;
  if (t1.pair) {  // each CTA of a pair loads 128 token rows and 128 weight rows per k-block
    MOE_TRY(make_a_maps(&m1, x, 2, P, H, 1, "stacked_expert_tokens"));
    MOE_TRY(make_tmap(&m1.b0, gate_w, 2, E * I, H, kBM, "gate_w"));
    MOE_TRY(make_tmap(&m1.b1, up_w, 2, E * I, H, kBM, "up_w"));
    m1.b1_row_offset = 0;
  } else {
    MOE_TRY(make_a_maps(&m1, x, 2, P, H, gmax1, "stacked_expert_tokens", t1.kpa));
    MOE_TRY(make_stage1_weights(&m1, gate_w, up_w, 2, E * I, H, t1, gate_w, up_w, E * I, 0, "gate_w/up_w"));
  }
  MOE_TRY(make_a_maps(&m2, U, 2, P, I, t2.pair ? 1 : gmax2, "workspace", t2.kpa));
  MOE_TRY(make_w_map(&m2.b0, down_w, 2, E * H, I, t2.pair ? kBM : (bn2 < kMmaN ? bn2 : kMmaN), t2.kpb, "down_w"));
  m2.b1 = m2.b0;

  if (gmax1 > 1 || gmax2 > 1) {  // pair each expert's blocks (from group_padded_offsets)
    build_groups_kernel<<<1, 1024, 0, s>>>(gpo, (int)E, 2, (int)nblk, groups, ngroups, done, single ? (int)nblk : 0);
    MOE_CUDA(cudaGetLastError());
  }

  GemmArgs a1{};
  a1.K = (int)H;
  a1.N = (int)I;
  a1.n_tiles = (int)((I + bn1 / 2 - 1) / (bn1 / 2));
  a1.ngroups = gmax1 > 1 ? -1 : (int)nblk;
  a1.ngroups_dev = ngroups;
  a1.groups = gmax1 > 1 ? groups : nullptr;
  a1.E = (int)E;
  a1.block_expert = gidx;
  a1.nblk = (int)nblk;
  a1.b_rows_per_expert = (int)I;
  a1.b1_row_offset = 0;
  a1.group_padded_offsets = gpo;
  a1.group_sizes = gs;
  a1.U = U;
  a1.ldu = (int)I;
  a1.status = status;

  GemmArgs a2 = a1;
  a2.K = (int)I;
  a2.N = (int)H;
  a2.n_tiles = (int)((H + bn2 - 1) / bn2);
  a2.ngroups = gmax2 > 1 ? -1 : (int)nblk;
  a2.groups = gmax2 > 1 ? groups : nullptr;
  a2.b_rows_per_expert = (int)H;
  a2.U = nullptr;
  a2.out = out;
  a2.ldo = (int)H;
  a2.group_sizes = gs;
  a2.group_offsets = go;
  a2.group_padded_offsets = gpo;
  a2.routed = routed;
  a2.routed_dtype = routed_dtype == MOE_F32 ? 0 : 1;
  a2.R = (int)R;

  a1.a_ptr = x;
  a1.a_row_bytes = H * 2;
  a2.a_ptr = U;
  a2.a_row_bytes = I * 2;
  const int tiles1 = (int)nblk * a1.n_tiles, tiles2 = (int)nblk * a2.n_tiles;
  if (single) {
    a1.block_done = a2.block_done = done;
    a1.block_done_target = a2.block_done_target = static_cast<uint32_t>(a1.n_tiles * 8);  // x 8 epilogue warps
    return launch_single_rt<kStage2Pad>(dtype, dev, m1, a1, m2, a2, tiles1, s);
  }
  MOE_TRY((launch_stage_rt<kStage1, false, kALsu>(dtype, lsu, tc1, dev, m1, a1, tiles1, s)));
  MOE_TRY((launch_stage_rt<kStage2Pad, false, kALsu>(dtype, lsu, tc2, dev, m2, a2, tiles2, s)));
  return MOE_OK;
}

// ---------------------------------------------------------------------------- run_kernel, no allocation
// The intermediate buffer for moe_run_kernel_noalloc: library-owned static device memory, so the
// call needs no caller workspace and allocates nothing. Host code must not use the symbol as a
// pointer (on the host it is only a stand-in); its device address is looked up per device.
static __device__ __align__(256) uint8_t g_noalloc_ws[MOE_NOALLOC_WORKSPACE_BYTES];
static std::atomic<void*> g_noalloc_ptr[kMaxDevices];

int moe_run_kernel_noalloc(const void* x, const void* gate_w, const void* up_w, const void* down_w,
                           const void* routed, int routed_dtype, const int32_t* gs, const int32_t* go,
                           const int32_t* gpo, const int32_t* gidx, void* out, int64_t P, int64_t H, int64_t I,
                           int64_t E, int64_t R, int64_t nblk, int dtype, void* stream) {
  t_last_error.clear();
  // the sizes are checked before the byte count is formed from them (no wrap-around of P * I)
  MOE_TRY(check_common(H, I, E, dtype, 8));
  if (P < 0 || P > (int64_t(1) << 31) - 1) return fail(MOE_ERR_INVALID_ARG, "total_padded_tokens out of range");
  const size_t need = moe_run_kernel_workspace_bytes(P, I, dtype);
  if (need > MOE_NOALLOC_WORKSPACE_BYTES)
    return fail(MOE_ERR_WORKSPACE,
                "moe_run_kernel_noalloc: this problem needs %zu bytes of intermediate storage, the static buffer "
                "holds %u (use moe_run_kernel with a caller workspace)",
                need, MOE_NOALLOC_WORKSPACE_BYTES);
  int dev;
  MOE_TRY(current_device(&dev));
  void* ptr = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (ptr == nullptr) {  // first call on this device: look up the buffer's device address
    MOE_CUDA(cudaGetSymbolAddress(&ptr, g_noalloc_ws));
    g_noalloc_ptr[dev].store(ptr, std::memory_order_release);
  }
  return moe_run_kernel(x, gate_w, up_w, down_w, routed, routed_dtype, gs, go, gpo, gidx, out, P, H, I, E, R, nblk,
                        dtype, ptr, MOE_NOALLOC_WORKSPACE_BYTES, stream);
}

// ---------------------------------------------------------------------------- align
int64_t moe_max_padded_rows(int64_t R, int64_t E, int64_t bm) {
  if (R <= 0 || E <= 0 || bm <= 0) return 0;
  const int64_t nonempty = R < E ? R : E;
  return (R + nonempty * (bm - 1) + bm - 1) / bm * bm;
}

size_t moe_align_workspace_bytes(int64_t R, int64_t E) {
  return round_up(sizeof(int) * static_cast<size_t>(align_chunks(R)) * static_cast<size_t>(E > 0 ? E : 0), 256);
}

int moe_router_grouped_topk(const void* logits, int logits_dtype, const float* bias, int64_t T, int64_t E,
                            int64_t n_group, int64_t topk_group, int64_t topk, int renormalize, float scale,
                            int32_t* ids, float* w, void* stream) {
  t_last_error.clear();
  if (logits_dtype != MOE_F32 && logits_dtype != MOE_F16 && logits_dtype != MOE_BF16)
    return fail(MOE_ERR_INVALID_ARG, "router logits must be fp32, fp16 or bf16");
  if (E < 1 || E > kAlignMaxExperts) return fail(MOE_ERR_INVALID_ARG, "num_experts must be in [1, %d]", kAlignMaxExperts);
  if (n_group < 1 || n_group > 32 || E % n_group != 0)
    return fail(MOE_ERR_INVALID_ARG, "num_expert_group must be in [1, 32] and divide num_experts");
  if (topk_group < 1 || topk_group > n_group) return fail(MOE_ERR_INVALID_ARG, "topk_group must be in [1, num_expert_group]");
  if (topk < 1 || topk > kRouterMaxTopk || topk > topk_group * (E / n_group))
    return fail(MOE_ERR_INVALID_ARG, "topk must be in [1, min(%d, topk_group * experts per group)]", kRouterMaxTopk);
  if (T < 0 || T * topk > (int64_t(1) << 31) - 1) return fail(MOE_ERR_INVALID_ARG, "bad token count");
  if (T == 0) return MOE_OK;
  if (!logits || !ids || !w) return fail(MOE_ERR_INVALID_ARG, "null tensor argument");
  int dev, sms;
  MOE_TRY(current_device(&dev));
  MOE_TRY(device_sms(dev, &sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rn = renormalize ? 1 : 0;
  if (logits_dtype == MOE_F32)
    return launch_router_grouped_t(static_cast<const float*>(logits), bias, T, E, n_group, topk_group, topk, rn, scale,
                                   ids, w, sms, s);
  if (logits_dtype == MOE_F16)
    return launch_router_grouped_t(static_cast<const __half*>(logits), bias, T, E, n_group, topk_group, topk, rn,
                                   scale, ids, w, sms, s);
  return launch_router_grouped_t(static_cast<const __nv_bfloat16*>(logits), bias, T, E, n_group, topk_group, topk, rn,
                                 scale, ids, w, sms, s);
}

int moe_router_topk(const void* logits, int logits_dtype, int64_t T, int64_t E, int64_t topk, int renormalize,
                    int32_t* ids, float* w, void* stream) {
  t_last_error.clear();
  MOE_TRY(check_router(logits, logits_dtype, T, E, topk, ids, w));
  if (T == 0) return MOE_OK;
  return launch_router(logits, logits_dtype, T, E, topk, renormalize, ids, w, nullptr,
                       static_cast<cudaStream_t>(stream));
}

int moe_align(const void* ids, int ids_dtype, int64_t R, int64_t E, int64_t bm, int32_t* gs, int32_t* go,
              int32_t* gpo, int32_t* gidx, int32_t* sorted, int32_t* route_slot, int32_t* meta, void* workspace,
              size_t workspace_bytes, void* stream) {
  t_last_error.clear();
  if (E < 1 || E > kAlignMaxExperts) return fail(MOE_ERR_INVALID_ARG, "num_experts must be in [1, %d]", kAlignMaxExperts);
  if (bm < 1 || bm > (1 << 20)) return fail(MOE_ERR_INVALID_ARG, "block_m must be in [1, 2^20]");
  if (R < 0 || moe_max_padded_rows(R, E, bm) > (int64_t(1) << 31) - 1) return fail(MOE_ERR_INVALID_ARG, "bad route count");
  if (ids_dtype != MOE_I32 && ids_dtype != MOE_I64) return fail(MOE_ERR_INVALID_ARG, "topk_ids must be int32 or int64");
  if (!gs || !go || !gpo || !sorted || !meta || (R > 0 && (!ids || !route_slot)))
    return fail(MOE_ERR_INVALID_ARG, "null output");
  if (R > 0 && (!workspace || workspace_bytes < moe_align_workspace_bytes(R, E)))
    return fail(MOE_ERR_WORKSPACE, "workspace must hold %zu bytes", moe_align_workspace_bytes(R, E));
  MOE_TRY(launch_align(ids, ids_dtype, R, E, bm, gs, go, gpo, gidx, sorted, route_slot, meta,
                       static_cast<int*>(workspace), static_cast<cudaStream_t>(stream)));
  return MOE_OK;
}

// ---------------------------------------------------------------------------- fused
size_t moe_fused_workspace_bytes(int64_t T, int64_t topk, int64_t E, int64_t H, int64_t I, int dtype) {
  (void)dtype;
  if (T <= 0 || topk <= 0 || E <= 0 || H <= 0 || I <= 0) return 0;
  return fused_layout(T, topk, E, H, I, false, a_path_lsu() || a_path_gather()).total;
}

// Expert parallelism over peer memory: token rows come from the ranks' regions (route r = (s *
// T_max + t) * topk + j reads row t of rank s) and `out` is this rank's partial-output block; the
// fused pipeline is otherwise unchanged.
struct PeerSource {
  const uint64_t* regions;
  EpRegion L;
  int rank, W, T_max;
  bool push;  // Stage2 adds into the home ranks' y rows instead of this rank's partial block
};

// Routing from router logits: the router kernel writes `ids` / `tw` (the fused call's topk_ids /
// topk_weights) and the alignment histogram.
struct RouterSource {
  const void* logits;
  int logits_dtype, renormalize;
};

static int fused_common(bool int8, const void* x, const void* w13, const float* w13_scale, const void* w2,
                        const float* w2_scale, const void* ids, int ids_dtype, const void* tw, int w_dtype, void* out,
                        int64_t T, int64_t H, int64_t I, int64_t E, int64_t topk, int dtype, void* workspace,
                        size_t workspace_bytes, void* stream, const PeerSource* peer = nullptr,
                        const RouterSource* router = nullptr, bool ordered = false, bool fp8 = false) {
  t_last_error.clear();
  MOE_TRY(check_common(H, I, E, dtype, int8 ? 16 : 8));
  if (T < 0 || topk < 1) return fail(MOE_ERR_INVALID_ARG, "num_tokens must be >= 0 and topk >= 1");
  if (E > kAlignMaxExperts) return fail(MOE_ERR_INVALID_ARG, "num_experts must be <= %d", kAlignMaxExperts);
  if (ids_dtype != MOE_I32 && ids_dtype != MOE_I64) return fail(MOE_ERR_INVALID_ARG, "topk_ids must be int32 or int64");
  if (w_dtype != MOE_F32 && w_dtype != MOE_F16 && w_dtype != MOE_BF16)
    return fail(MOE_ERR_INVALID_ARG, "topk_weights must be fp32, fp16 or bf16");
  if (T == 0) return MOE_OK;
  const int64_t R = T * topk;
  if (moe_max_padded_rows(R, E, kBM) > (int64_t(1) << 31) - 1 || 2 * E * I > (int64_t(1) << 31) - 1 ||
      E * H > (int64_t(1) << 31) - 1)
    return fail(MOE_ERR_INVALID_ARG, "problem exceeds 32-bit row indexing");
  if (!x || !w13 || !w2 || !ids || !tw || !out) return fail(MOE_ERR_INVALID_ARG, "null tensor argument");
  if (int8 && (!w13_scale || !w2_scale)) return fail(MOE_ERR_INVALID_ARG, "null weight scales");
  if (!aligned16(x) || !aligned16(out)) return fail(MOE_ERR_ALIGNMENT, "hidden_states/out must be 16-byte aligned");
  if (peer && int8) return fail(MOE_ERR_UNSUPPORTED, "the int8 route has no peer-memory expert-parallel mode");
  const bool lsu = a_path_lsu() && !peer;
  // tile::gather4 A path: Stage1 reads the token rows in place (peer mode stages them itself)
  const bool gather = a_path_gather() && !peer;
  if (ordered && (int8 || peer)) return fail(MOE_ERR_UNSUPPORTED, "the ordered combine is for the fp16/bf16 route");
  if (fp8 && !int8) return fail(MOE_ERR_INVALID_ARG, "fp8 is an 8-bit route");
  if (fp8 && lsu) return fail(MOE_ERR_UNSUPPORTED, "the fp8 route runs on the TMA A path (MOE_B200_A_PATH=tma)");
  const FusedLayout L = fused_layout(T, topk, E, H, I, int8, lsu || gather, ordered);
  if (!workspace || workspace_bytes < L.total) return fail(MOE_ERR_WORKSPACE, "workspace must hold %zu bytes", L.total);
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return fail(MOE_ERR_ALIGNMENT, "workspace must be 256-byte aligned");

  int dev;
  MOE_TRY(current_device(&dev));
  uint32_t* status;
  MOE_TRY(device_status_ptr(dev, &status));
  int sms;
  MOE_TRY(device_sms(dev, &sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* counts = reinterpret_cast<int*>(ws + L.counts);
  int32_t* gs = reinterpret_cast<int32_t*>(ws + L.gs);
  int32_t* go = reinterpret_cast<int32_t*>(ws + L.go);
  int32_t* gpo = reinterpret_cast<int32_t*>(ws + L.gpo);
  int32_t* meta = reinterpret_cast<int32_t*>(ws + L.meta);
  int32_t* gidx = reinterpret_cast<int32_t*>(ws + L.gidx);
  int32_t* sorted = reinterpret_cast<int32_t*>(ws + L.sorted);
  int32_t* slot = reinterpret_cast<int32_t*>(ws + L.slot);
  void* xs = ws + L.xs;
  void* U = ws + L.u;
  int32_t* groups = reinterpret_cast<int32_t*>(ws + L.groups);
  int32_t* ngroups = groups + L.nblk_max;
  uint32_t* done = reinterpret_cast<uint32_t*>(ws + L.done);
  const int elt = int8 ? 1 : 2;
  // expected blocks per expert: routes per expert / 128, plus half a block of padding (peer mode:
  // about 1 / W of the virtual routes land on this rank)
  const double bpe = static_cast<double>(R) / (peer ? peer->W : 1) / static_cast<double>(E) / kBM + 0.5;
  TileCfg tc1 = usable_cfg(1, H, elt, lsu, bpe);
  TileCfg tc2 = usable_cfg(2, I, elt, lsu, bpe);
  // the push combine runs its Stage2 on the single-CTA kernel: with the CTA-pair kernel it timed
  // out at the bench's size while the single-CTA form passed its parity tests
  if (peer && peer->push && kTiles[tc2].pair) tc2 = kDefaultTile2;
  if (gather && !gather_cfg(tc1)) tc1 = kDefaultTile1;
  // single-kernel MoE: both stages in one launch, on their default single-CTA tiles
  const bool single = single_kernel(bpe) && !int8 && !peer && !lsu && !gather && !ordered &&
                      tile_cfg(1) == kAuto && tile_cfg(2) == kAuto;
  if (single) {
    tc1 = kDefaultTile1;
    tc2 = kDefaultTile2;
  }
  // peer memory with the fused token gather: Stage1's gather warps copy the routed rows from the
  // peers' regions while its weights stream (Stage1 on its default tile)
  const bool fused_gather = peer && ep_gather_mode() == kEpGatherFused && !int8 && tc1 == kDefaultTile1;
  const TileInfo &t1 = kTiles[tc1], &t2 = kTiles[tc2];
  if (peer && peer->push && t2.tn) return fail(MOE_ERR_UNSUPPORTED, "the operand-swapped Stage2 has no push combine");
  const int bn1 = t1.bn, gmax1 = t1.gmax, bn2 = t2.bn, gmax2 = t2.gmax;

  // 1. routing metadata
  prof_record(0, s);
  if (router)
    MOE_TRY(launch_router(router->logits, router->logits_dtype, T, E, topk, router->renormalize,
                          static_cast<int32_t*>(const_cast<void*>(ids)), static_cast<float*>(const_cast<void*>(tw)),
                          counts, s));
  MOE_TRY(launch_align(ids, ids_dtype, R, E, kBM, gs, go, gpo, gidx, sorted, slot, meta, counts, s, router != nullptr));
  if (gmax1 > 1 || gmax2 > 1 || single || fused_gather) {  // also clears the per-block counts
    build_groups_kernel<<<1, 1024, 0, s>>>(gpo, (int)E, 2, (int)L.nblk_max, groups, ngroups, done,
                                           fused_gather ? (int)(L.nblk_max + T) : single ? (int)L.nblk_max : 0);
    MOE_CUDA(cudaGetLastError());
  }
  int32_t* tn_entries = reinterpret_cast<int32_t*>(ws + L.tn);
  int32_t* tn_count = tn_entries + 2 * L.nblk_max;
  if (t1.tn || t2.tn) {  // (expert, token chunk) entries of the operand-swapped kernel
    build_tn_entries_kernel<<<1, 1024, 0, s>>>(gs, (int)E, (int)L.nblk_max, tn_entries, tn_count);
    MOE_CUDA(cudaGetLastError());
  }
  prof_record(1, s);

  // 2. activations: the TMA A path stacks the gathered token rows (int8: quantised per token)
  //    and zeroes the combine target; the LSU path gathers token rows inside Stage1 (int8: after
  //    an in-place per-token quantisation) and Stage1's epilogue warps zero the combine target
  const int gblocks = sms * 4;
  float* amax = int8 ? reinterpret_cast<float*>(ws + L.amax) : nullptr;
  float* xscale = int8 ? reinterpret_cast<float*>(ws + L.xscale) : nullptr;
  if (lsu || gather) {
    if (int8) {  // quantised per token, once (each token's k routes share its row and scale)
      if (dtype == MOE_F16 && fp8)
        quantize_rows_q8_kernel<__half, kQF8><<<gblocks, 256, 0, s>>>(
            static_cast<const __half*>(x), T, (int)H, nullptr, nullptr, static_cast<int8_t*>(xs), xscale);
      else if (dtype == MOE_F16)
        quantize_rows_q8_kernel<__half><<<gblocks, 256, 0, s>>>(static_cast<const __half*>(x), T, (int)H, nullptr,
                                                                nullptr, static_cast<int8_t*>(xs), xscale);
      else if (fp8)
        quantize_rows_q8_kernel<__nv_bfloat16, kQF8><<<gblocks, 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(x), T, (int)H, nullptr, nullptr, static_cast<int8_t*>(xs), xscale);
      else
        quantize_rows_q8_kernel<__nv_bfloat16><<<gblocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), T,
                                                                       (int)H, nullptr, nullptr,
                                                                       static_cast<int8_t*>(xs), xscale);
      MOE_CUDA(cudaGetLastError());
      MOE_CUDA(cudaMemsetAsync(amax, 0, sizeof(float) * (size_t)L.P_max, s));
    }
  } else if (fused_gather) {
    // the token rows are copied by Stage1's gather warps, which also zero the served partial rows
  } else if (peer && ep_gather_mode() == kEpGatherDedup && topk <= 32) {
    // one warp per virtual token: its row crosses NVLink once, then lands in all its local slots
    const int zero_served = peer->push ? 0 : 1;
    if (dtype == MOE_F16)
      gather_rows_peer_dedup_kernel<__half><<<gblocks, 256, 0, s>>>(peer->regions, peer->L, peer->rank,
                                                                    peer->T_max, (int)topk, peer->W, slot, (int)H,
                                                                    static_cast<__half*>(xs), zero_served);
    else
      gather_rows_peer_dedup_kernel<__nv_bfloat16><<<gblocks, 256, 0, s>>>(
          peer->regions, peer->L, peer->rank, peer->T_max, (int)topk, peer->W, slot, (int)H,
          static_cast<__nv_bfloat16*>(xs), zero_served);
    MOE_CUDA(cudaGetLastError());
  } else if (peer && ep_gather_mode() == kEpGatherBulk &&
             (size_t)kEpBulkWarps * 2 * (size_t)H * 2 + 16 * kEpBulkWarps <= kEpBulkMaxSmem) {
    // bulk-copy gather: whole rows through shared memory, one CTA of 4 warps per SM
    const size_t smem = (size_t)kEpBulkWarps * 2 * (size_t)H * 2 + 16 * kEpBulkWarps;
    const int zero_served = peer->push ? 0 : 1;
    if (dtype == MOE_F16) {
      MOE_CUDA(cudaFuncSetAttribute(gather_rows_peer_bulk_kernel<__half>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      gather_rows_peer_bulk_kernel<__half><<<sms, kEpBulkWarps * 32, smem, s>>>(
          peer->regions, peer->L, peer->rank, peer->T_max, (int)topk, peer->W, slot,
          static_cast<const int32_t*>(ids), (int)H, static_cast<__half*>(xs), status, zero_served);
    } else {
      MOE_CUDA(cudaFuncSetAttribute(gather_rows_peer_bulk_kernel<__nv_bfloat16>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      gather_rows_peer_bulk_kernel<__nv_bfloat16><<<sms, kEpBulkWarps * 32, smem, s>>>(
          peer->regions, peer->L, peer->rank, peer->T_max, (int)topk, peer->W, slot,
          static_cast<const int32_t*>(ids), (int)H, static_cast<__nv_bfloat16*>(xs), status, zero_served);
    }
    MOE_CUDA(cudaGetLastError());
  } else if (peer) {  // token rows from the ranks' regions; zero the served partial rows
    const int zero_served = peer->push ? 0 : 1;
    if (dtype == MOE_F16)
      gather_rows_peer_kernel<__half><<<gblocks, 256, 0, s>>>(peer->regions, peer->L, peer->rank, peer->T_max,
                                                              (int)topk, peer->W, slot, static_cast<const int32_t*>(ids),
                                                              (int)H, static_cast<__half*>(xs), zero_served);
    else
      gather_rows_peer_kernel<__nv_bfloat16><<<gblocks, 256, 0, s>>>(
          peer->regions, peer->L, peer->rank, peer->T_max, (int)topk, peer->W, slot,
          static_cast<const int32_t*>(ids), (int)H, static_cast<__nv_bfloat16*>(xs), zero_served);
    MOE_CUDA(cudaGetLastError());
  } else if (dtype == MOE_F16) {
    if (fp8)
      gather_rows_q8_kernel<__half, kQF8><<<gblocks, 256, 0, s>>>(
          static_cast<const __half*>(x), slot, (int)R, (int)topk, (int)H, static_cast<int8_t*>(xs), xscale,
          static_cast<__half*>(out), (int)T, amax, (int)L.P_max);
    else if (int8)
      gather_rows_q8_kernel<__half><<<gblocks, 256, 0, s>>>(static_cast<const __half*>(x), slot, (int)R, (int)topk,
                                                            (int)H, static_cast<int8_t*>(xs), xscale,
                                                            static_cast<__half*>(out), (int)T, amax, (int)L.P_max);
    else
      gather_rows_kernel<__half><<<gblocks, 256, 0, s>>>(static_cast<const __half*>(x), slot, (int)R, (int)topk,
                                                         (int)H, static_cast<__half*>(xs), static_cast<__half*>(out),
                                                         ordered ? 0 : (int)T, nullptr, 0);
    MOE_CUDA(cudaGetLastError());
  } else {
    if (fp8)
      gather_rows_q8_kernel<__nv_bfloat16, kQF8><<<gblocks, 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), slot, (int)R, (int)topk, (int)H, static_cast<int8_t*>(xs), xscale,
          static_cast<__nv_bfloat16*>(out), (int)T, amax, (int)L.P_max);
    else if (int8)
      gather_rows_q8_kernel<__nv_bfloat16><<<gblocks, 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), slot, (int)R, (int)topk, (int)H, static_cast<int8_t*>(xs), xscale,
          static_cast<__nv_bfloat16*>(out), (int)T, amax, (int)L.P_max);
    else
      gather_rows_kernel<__nv_bfloat16><<<gblocks, 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), slot, (int)R, (int)topk, (int)H, static_cast<__nv_bfloat16*>(xs),
          static_cast<__nv_bfloat16*>(out), ordered ? 0 : (int)T, nullptr, 0);
    MOE_CUDA(cudaGetLastError());
  }
  prof_record(2, s);

  // 3. Stage1 (gate/up GEMM + SiLU*up) and 4. Stage2 (down GEMM * topk weight, combine)
  const void* a1_src = (lsu || gather) ? (int8 ? static_cast<const void*>(xs) : x) : xs;
  void* a2_src = int8 ? (void*)(ws + L.uq) : U;
  StageMaps m1, m2;
  const uint8_t* w13b = static_cast<const uint8_t*>(w13);
  if (t1.pair) {  // gate rows and up rows (at +I) of the stacked weights, 128-row boxes
    MOE_TRY(make_tmap(&m1.b0, w13, elt, 2 * E * I, H, kBM, "w_gate_up"));
    m1.b1 = m1.b0;
    m1.b1_row_offset = (int)I;
  } else {
    MOE_TRY(make_stage1_weights(&m1, w13, w13b + static_cast<size_t>(I) * H * elt, elt, 2 * E * I - I, H, t1, w13,
                                w13, 2 * E * I, (int)I, "w_gate_up"));
  }
  MOE_TRY(make_w_map(&m2.b0, w2, elt, E * H, I, t2.pair ? kBM : (bn2 < kMmaN ? bn2 : kMmaN), t2.kpb, "w_down"));
  m2.b1 = m2.b0;
  if (lsu) {  // the LSU path does not use the A tensor maps
    m1.a = m1.a1 = m1.b0;
    m2.a = m2.a1 = m2.b0;
    if (ordered) MOE_TRY(make_a_maps(&m2, a2_src, elt, L.P_max, I, t2.pair ? 1 : gmax2, "intermediate", t2.kpa));
  } else if (gather) {  // Stage1: the token rows themselves, boxes one row high (tile::gather4)
    MOE_TRY(make_tmap(&m1.a, a1_src, elt, T, H, 1, "hidden_states (gather4)"));
    m1.a1 = m1.a;
    MOE_TRY(make_a_maps(&m2, a2_src, elt, L.P_max, I, t2.pair ? 1 : gmax2, "intermediate", t2.kpa));
  } else {
    MOE_TRY(make_a_maps(&m1, xs, elt, L.P_max, H, t1.pair ? 1 : gmax1, "gathered hidden_states", t1.kpa));
    MOE_TRY(make_a_maps(&m2, a2_src, elt, L.P_max, I, t2.pair ? 1 : gmax2, "intermediate", t2.kpa));
  }

  GemmArgs a1{};
  a1.K = (int)H;
  a1.N = (int)I;
  a1.n_tiles = (int)((I + bn1 / 2 - 1) / (bn1 / 2));
  a1.ngroups = -1;
  a1.ngroups_dev = gmax1 > 1 ? ngroups : meta + 1;
  a1.groups = gmax1 > 1 ? groups : nullptr;
  a1.E = (int)E;
  a1.block_expert = gidx;
  a1.nblk = (int)L.nblk_max;
  a1.b_rows_per_expert = (int)(2 * I);
  a1.b1_row_offset = (int)I;
  a1.group_padded_offsets = gpo;
  a1.group_sizes = gs;
  a1.U = U;
  a1.ldu = (int)I;
  a1.a_scale = xscale;
  a1.b0_scale = w13_scale;
  a1.b1_scale = w13_scale;
  a1.row_amax = amax;
  a1.status = status;
  a1.a_ptr = a1_src;
  a1.a_row_bytes = H * elt;
  a1.sorted_route_ids = sorted;
  a1.R = (int)R;
  a1.topk = (int)topk;
  a1.zero_ptr = (lsu || gather) && !ordered ? out : nullptr;
  a1.zero_bytes = (lsu || gather) && !ordered ? T * H * 2 : 0;

  GemmArgs a2{};
  a2.K = (int)I;
  a2.N = (int)H;
  a2.n_tiles = (int)((H + bn2 - 1) / bn2);
  a2.ngroups = -1;
  a2.ngroups_dev = gmax2 > 1 ? ngroups : meta + 1;
  a2.groups = gmax2 > 1 ? groups : nullptr;
  a2.E = (int)E;
  a2.block_expert = gidx;
  a2.nblk = (int)L.nblk_max;
  a2.b_rows_per_expert = (int)H;
  a2.group_padded_offsets = gpo;
  a2.group_sizes = gs;
  a2.out = out;
  a2.ldo = (int)H;
  a2.routed = tw;
  a2.routed_dtype = w_dtype == MOE_F32 ? 0 : (w_dtype == MOE_F16 ? 1 : 2);
  a2.R = (int)R;
  a2.sorted_route_ids = sorted;
  a2.topk = (int)topk;
  a2.a_scale = int8 ? reinterpret_cast<const float*>(ws + L.uscale) : nullptr;
  a2.b0_scale = w2_scale;
  a2.status = status;
  a2.a_ptr = a2_src;
  a2.a_row_bytes = I * elt;
  if (peer && peer->push) {  // push combine: Stage2 adds into the home ranks' y rows
    a2.out_regions = peer->regions;
    a2.out_region_off = peer->L.y;
    a2.out_T_max = peer->T_max;
  }

  const int max_tiles1 = (int)L.nblk_max * a1.n_tiles, max_tiles2 = (int)L.nblk_max * a2.n_tiles;
  // the operand-swapped kernel (tile "tn"): weights as the MMA's M side, tokens as N
  TnArgs tn{};
  tn.n_entries_dev = tn_count;
  tn.entries = tn_entries;
  tn.E = (int)E;
  tn.group_sizes = gs;
  tn.group_offsets = go;
  tn.group_padded_offsets = gpo;
  tn.R = (int)R;
  tn.sorted_route_ids = sorted;
  tn.topk = (int)topk;
  tn.nblk = (int)L.nblk_max;
  tn.status = status;
  if (!int8) {
    if (t1.tn) {
      TnMaps tm{};
      MOE_TRY(make_tn_w13_map(&tm.w, w13, 2, E, H, I));
      MOE_TRY(make_tn_x_maps(&tm, xs, 2, L.P_max, H, "gathered hidden_states"));
      TnArgs t = tn;
      t.K = (int)H;
      t.N = (int)I;
      t.n_tiles = (int)((I + 63) / 64);
      t.w_group_per_expert = 2 * I / 8;
      t.U = U;
      t.ldu = (int)I;
      MOE_TRY(launch_tn_rt<kStage1>(dtype, dev, tc1, tm, t, (int)L.nblk_max * t.n_tiles, s));
    } else if (gather) {
      MOE_TRY(launch_stage1_gather_rt<kQ16>(dtype, tc1, dev, m1, a1, max_tiles1, s));
    } else if (fused_gather) {
      a1.g_regions = peer->regions;
      a1.g_x_off = peer->L.x;
      a1.g_T_max = peer->T_max;
      a1.g_rows = xs;
      a1.a_done = done;
      a1.g_zero_y = peer->push ? nullptr : out;
      a1.g_route_slot = slot;
      a1.g_tokens = (int)T;
      a1.g_claim = done + L.nblk_max;
      if (dtype == MOE_F16)
        MOE_TRY(launch_stage1_gather_warps<__half>(dev, m1, a1, max_tiles1, s));
      else
        MOE_TRY(launch_stage1_gather_warps<__nv_bfloat16>(dev, m1, a1, max_tiles1, s));
    } else if (single) {  // Stage1 and Stage2 in one launch: the Stage1 event marks the end of both
      a1.block_done = a2.block_done = done;
      a1.block_done_target = a2.block_done_target = static_cast<uint32_t>(a1.n_tiles * 8);  // x 8 epilogue warps
      MOE_TRY(launch_single_rt<kStage2Comb>(dtype, dev, m1, a1, m2, a2, max_tiles1, s));
    } else {
      MOE_TRY((launch_stage_rt<kStage1, false, kAGather>(dtype, lsu, tc1, dev, m1, a1, max_tiles1, s)));
    }
    prof_record(3, s);
    if (ordered) {
      // padded-store Stage2 into y (weights in raw order), then the in-order per-token sum
      if (t2.tn) return fail(MOE_ERR_UNSUPPORTED, "the operand-swapped Stage2 has no ordered combine");
      float* raw = reinterpret_cast<float*>(ws + L.raw);
      void* y = ws + L.y;
      raw_weights_kernel<<<sms * 2, 256, 0, s>>>(tw, a2.routed_dtype, sorted, gidx, go, gpo, meta, (int)R, L.P_max,
                                                 kBM, raw);
      MOE_CUDA(cudaGetLastError());
      GemmArgs a = a2;
      a.out = y;
      a.group_sizes = gs;
      a.group_offsets = go;
      a.routed = raw;
      a.routed_dtype = 0;
      MOE_TRY((launch_stage_rt<kStage2Pad, false, kALsu>(dtype, false, tc2, dev, m2, a, max_tiles2, s)));
      const int64_t want = (T + 7) / 8;
      const int cblocks = static_cast<int>(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
      if (dtype == MOE_F16)
        combine_ordered_kernel<__half><<<cblocks, 256, 0, s>>>(static_cast<const __half*>(y), slot, (int)T,
                                                               (int)topk, (int)H, static_cast<__half*>(out));
      else
        combine_ordered_kernel<__nv_bfloat16><<<cblocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(y), slot,
                                                                      (int)T, (int)topk, (int)H,
                                                                      static_cast<__nv_bfloat16*>(out));
      MOE_CUDA(cudaGetLastError());
    } else if (t2.tn) {
      TnMaps tm{};
      MOE_TRY(make_tmap(&tm.w, w2, 2, E * H, I, kBM, "w_down"));
      MOE_TRY(make_tn_x_maps(&tm, U, 2, L.P_max, I, "intermediate"));
      TnArgs t = tn;
      t.K = (int)I;
      t.N = (int)H;
      t.n_tiles = (int)((H + kBM - 1) / kBM);
      t.b_rows_per_expert = (int)H;
      t.out = out;
      t.ldo = (int)H;
      t.routed = tw;
      t.routed_dtype = w_dtype == MOE_F32 ? 0 : (w_dtype == MOE_F16 ? 1 : 2);
      MOE_TRY(launch_tn_rt<kStage2Comb>(dtype, dev, tc2, tm, t, (int)L.nblk_max * t.n_tiles, s));
    } else if (!single) {
      MOE_TRY((launch_stage_rt<kStage2Comb, false, kALsu>(dtype, lsu, tc2, dev, m2, a2, max_tiles2, s)));
    }
    prof_record(4, s);
  } else {
    // 8-bit routes (int8; fp8 with e4m3 operands, fp32 accumulation, TMA A path only): Stage1
    // writes U (16-bit) and its per-row amax; the rows are re-quantised for Stage2
    auto run8 = [&](auto kind) -> int {
      constexpr int Q = decltype(kind)::value;
      if (t1.tn) {
        TnMaps tm{};
        MOE_TRY(make_tn_w13_map(&tm.w, w13, 1, E, H, I));
        MOE_TRY(make_tn_x_maps(&tm, xs, 1, L.P_max, H, "quantised hidden_states"));
        TnArgs t = tn;
        t.K = (int)H;
        t.N = (int)I;
        t.n_tiles = (int)((I + 63) / 64);
        t.w_group_per_expert = 2 * I / 8;
        t.U = U;
        t.ldu = (int)I;
        t.a_scale = xscale;
        t.b_scale = w13_scale;
        t.b_scale_rows = (int)(2 * I);
        t.b_up_offset = (int)I;
        t.row_amax = amax;
        MOE_TRY((launch_tn_rt<kStage1, Q>(dtype, dev, tc1, tm, t, (int)L.nblk_max * t.n_tiles, s)));
      } else if (gather) {
        MOE_TRY(launch_stage1_gather_rt<Q>(dtype, tc1, dev, m1, a1, max_tiles1, s));
      } else if constexpr (Q == kQF8) {
        MOE_TRY((launch_stage_rt<kStage1, kQF8, kATma>(dtype, false, tc1, dev, m1, a1, max_tiles1, s)));
      } else {
        MOE_TRY((launch_stage_rt<kStage1, kQI8, kAGather>(dtype, lsu, tc1, dev, m1, a1, max_tiles1, s)));
      }
      prof_record(3, s);
      if (dtype == MOE_F16)
        quantize_rows_q8_kernel<__half, Q><<<sms * 4, 256, 0, s>>>(
            static_cast<const __half*>(U), L.P_max, (int)I, meta, amax, reinterpret_cast<int8_t*>(ws + L.uq),
            reinterpret_cast<float*>(ws + L.uscale));
      else
        quantize_rows_q8_kernel<__nv_bfloat16, Q><<<sms * 4, 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(U), L.P_max, (int)I, meta, amax, reinterpret_cast<int8_t*>(ws + L.uq),
            reinterpret_cast<float*>(ws + L.uscale));
      MOE_CUDA(cudaGetLastError());
      prof_record(4, s);
      if (t2.tn) {
        TnMaps tm{};
        MOE_TRY(make_tmap(&tm.w, w2, 1, E * H, I, kBM, "w_down"));
        MOE_TRY(make_tn_x_maps(&tm, ws + L.uq, 1, L.P_max, I, "quantised intermediate"));
        TnArgs t = tn;
        t.K = (int)I;
        t.N = (int)H;
        t.n_tiles = (int)((H + kBM - 1) / kBM);
        t.b_rows_per_expert = (int)H;
        t.out = out;
        t.ldo = (int)H;
        t.routed = tw;
        t.routed_dtype = w_dtype == MOE_F32 ? 0 : (w_dtype == MOE_F16 ? 1 : 2);
        t.a_scale = reinterpret_cast<const float*>(ws + L.uscale);
        t.b_scale = w2_scale;
        t.b_scale_rows = (int)H;
        MOE_TRY((launch_tn_rt<kStage2Comb, Q>(dtype, dev, tc2, tm, t, (int)L.nblk_max * t.n_tiles, s)));
      } else if constexpr (Q == kQF8) {
        MOE_TRY((launch_stage_rt<kStage2Comb, kQF8, kATma>(dtype, false, tc2, dev, m2, a2, max_tiles2, s)));
      } else {
        MOE_TRY((launch_stage_rt<kStage2Comb, kQI8, kALsu>(dtype, lsu, tc2, dev, m2, a2, max_tiles2, s)));
      }
      prof_record(5, s);
      return MOE_OK;
    };
    MOE_TRY(fp8 ? run8(std::integral_constant<int, kQF8>{}) : run8(std::integral_constant<int, kQI8>{}));
  }
  return MOE_OK;
}

int moe_fused(const void* x, const void* w13, const void* w2, const void* ids, int ids_dtype, const void* tw,
              int w_dtype, void* out, int64_t T, int64_t H, int64_t I, int64_t E, int64_t topk, int dtype,
              void* workspace, size_t workspace_bytes, void* stream) {
  return fused_common(false, x, w13, nullptr, w2, nullptr, ids, ids_dtype, tw, w_dtype, out, T, H, I, E, topk, dtype,
                      workspace, workspace_bytes, stream);
}

size_t moe_fused_ordered_workspace_bytes(int64_t T, int64_t topk, int64_t E, int64_t H, int64_t I, int dtype) {
  (void)dtype;
  if (T <= 0 || topk <= 0 || E <= 0 || H <= 0 || I <= 0) return 0;
  return fused_layout(T, topk, E, H, I, false, a_path_lsu() || a_path_gather(), true).total;
}

int moe_fused_ordered(const void* x, const void* w13, const void* w2, const void* ids, int ids_dtype, const void* tw,
                      int w_dtype, void* out, int64_t T, int64_t H, int64_t I, int64_t E, int64_t topk, int dtype,
                      void* workspace, size_t workspace_bytes, void* stream) {
  return fused_common(false, x, w13, nullptr, w2, nullptr, ids, ids_dtype, tw, w_dtype, out, T, H, I, E, topk, dtype,
                      workspace, workspace_bytes, stream, nullptr, nullptr, true);
}

int moe_fused_router(const void* x, const void* w13, const void* w2, const void* logits, int logits_dtype,
                     int renormalize, int32_t* ids, float* tw, void* out, int64_t T, int64_t H, int64_t I, int64_t E,
                     int64_t topk, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  t_last_error.clear();
  MOE_TRY(check_router(logits, logits_dtype, T, E, topk, ids, tw));
  const RouterSource rs{logits, logits_dtype, renormalize ? 1 : 0};
  return fused_common(false, x, w13, nullptr, w2, nullptr, ids, MOE_I32, tw, MOE_F32, out, T, H, I, E, topk, dtype,
                      workspace, workspace_bytes, stream, nullptr, &rs);
}

static int quantize_rows(bool fp8, const void* w, int dtype, int64_t rows, int64_t cols, void* q, float* scale,
                         void* stream) {
  t_last_error.clear();
  if (dtype != MOE_F16 && dtype != MOE_BF16) return fail(MOE_ERR_INVALID_ARG, "dtype must be MOE_F16 or MOE_BF16");
  if (rows < 0 || cols <= 0 || cols % 16 != 0) return fail(MOE_ERR_INVALID_ARG, "cols must be a positive multiple of 16");
  if (rows == 0) return MOE_OK;
  if (!w || !q || !scale) return fail(MOE_ERR_INVALID_ARG, "null tensor argument");
  if (!aligned16(w) || !aligned16(q)) return fail(MOE_ERR_ALIGNMENT, "w and q must be 16-byte aligned");
  int dev, sms;
  MOE_TRY(current_device(&dev));
  MOE_TRY(device_sms(dev, &sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (fp8 && dtype == MOE_F16)
    quantize_rows_q8_kernel<__half, kQF8><<<sms * 4, 256, 0, s>>>(static_cast<const __half*>(w), rows, (int)cols,
                                                                  nullptr, nullptr, static_cast<int8_t*>(q), scale);
  else if (fp8)
    quantize_rows_q8_kernel<__nv_bfloat16, kQF8><<<sms * 4, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(w), rows, (int)cols, nullptr, nullptr, static_cast<int8_t*>(q), scale);
  else if (dtype == MOE_F16)
    quantize_rows_q8_kernel<__half><<<sms * 4, 256, 0, s>>>(static_cast<const __half*>(w), rows, (int)cols, nullptr,
                                                            nullptr, static_cast<int8_t*>(q), scale);
  else
    quantize_rows_q8_kernel<__nv_bfloat16><<<sms * 4, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w), rows,
                                                                   (int)cols, nullptr, nullptr,
                                                                   static_cast<int8_t*>(q), scale);
  MOE_CUDA(cudaGetLastError());
  return MOE_OK;
}

int moe_quantize_rows_int8(const void* w, int dtype, int64_t rows, int64_t cols, void* q, float* scale, void* stream) {
  return quantize_rows(false, w, dtype, rows, cols, q, scale, stream);
}

int moe_quantize_rows_fp8(const void* w, int dtype, int64_t rows, int64_t cols, void* q, float* scale, void* stream) {
  return quantize_rows(true, w, dtype, rows, cols, q, scale, stream);
}

size_t moe_fused_int8_workspace_bytes(int64_t T, int64_t topk, int64_t E, int64_t H, int64_t I, int dtype) {
  (void)dtype;
  if (T <= 0 || topk <= 0 || E <= 0 || H <= 0 || I <= 0) return 0;
  return fused_layout(T, topk, E, H, I, true, a_path_lsu() || a_path_gather()).total;
}

int moe_fused_int8(const void* x, const void* w13_q, const float* w13_scale, const void* w2_q, const float* w2_scale,
                   const void* ids, int ids_dtype, const void* tw, int w_dtype, void* out, int64_t T, int64_t H,
                   int64_t I, int64_t E, int64_t topk, int dtype, void* workspace, size_t workspace_bytes,
                   void* stream) {
  return fused_common(true, x, w13_q, w13_scale, w2_q, w2_scale, ids, ids_dtype, tw, w_dtype, out, T, H, I, E, topk,
                      dtype, workspace, workspace_bytes, stream);
}

size_t moe_fused_fp8_workspace_bytes(int64_t T, int64_t topk, int64_t E, int64_t H, int64_t I, int dtype) {
  (void)dtype;
  if (T <= 0 || topk <= 0 || E <= 0 || H <= 0 || I <= 0) return 0;
  return fused_layout(T, topk, E, H, I, true, a_path_gather()).total;
}

int moe_fused_fp8(const void* x, const void* w13_q, const float* w13_scale, const void* w2_q, const float* w2_scale,
                  const void* ids, int ids_dtype, const void* tw, int w_dtype, void* out, int64_t T, int64_t H,
                  int64_t I, int64_t E, int64_t topk, int dtype, void* workspace, size_t workspace_bytes,
                  void* stream) {
  return fused_common(true, x, w13_q, w13_scale, w2_q, w2_scale, ids, ids_dtype, tw, w_dtype, out, T, H, I, E, topk,
                      dtype, workspace, workspace_bytes, stream, nullptr, nullptr, false, true);
}

// ---------------------------------------------------------------------------- packed weights
// One buffer per expert set: w13 [E, 2I, H], w13 scales, w2 [E, H, I], w2 scales, each section
// 256-byte aligned (include/moe_b200.h gives the contract).
static bool packed_q8(int kind) { return kind == MOE_I8 || kind == MOE_F8E4M3; }

int moe_packed_weights_layout(int64_t E, int64_t H, int64_t I, int kind, size_t offsets[4], size_t* total_bytes) {
  t_last_error.clear();
  if (kind != MOE_F16 && kind != MOE_BF16 && !packed_q8(kind))
    return fail(MOE_ERR_INVALID_ARG, "kind must be MOE_F16, MOE_BF16, MOE_I8 or MOE_F8E4M3");
  if (E < 1 || E > kAlignMaxExperts || H < 1 || I < 1 || H > (1 << 30) || I > (1 << 30))
    return fail(MOE_ERR_INVALID_ARG, "bad packed weight shape");
  const bool q = packed_q8(kind);
  const size_t elt = q ? 1 : 2;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t r = o;
    o = round_up(o + bytes, 256);
    return r;
  };
  size_t off[4];
  off[0] = take(static_cast<size_t>(E) * 2 * I * H * elt);
  off[1] = take(q ? sizeof(float) * E * 2 * I : 0);
  off[2] = take(static_cast<size_t>(E) * H * I * elt);
  off[3] = take(q ? sizeof(float) * E * H : 0);
  if (offsets)
    for (int i = 0; i < 4; ++i) offsets[i] = off[i];
  if (total_bytes) *total_bytes = o;
  return MOE_OK;
}

int moe_pack_weights(const void* gate_w, const void* up_w, const void* down_w, int dtype, int64_t E, int64_t H,
                     int64_t I, int kind, void* packed, size_t packed_bytes, void* stream) {
  size_t off[4], total;
  MOE_TRY(moe_packed_weights_layout(E, H, I, kind, off, &total));
  const bool q = packed_q8(kind);
  MOE_TRY(check_common(H, I, E, dtype, q ? 16 : 8));
  if (!q && kind != dtype) return fail(MOE_ERR_INVALID_ARG, "16-bit packing keeps the weights' dtype");
  if (!gate_w || !up_w || !down_w || !packed) return fail(MOE_ERR_INVALID_ARG, "null tensor argument");
  if (packed_bytes < total) return fail(MOE_ERR_INVALID_ARG, "packed must hold %zu bytes", total);
  if (!aligned16(gate_w) || !aligned16(up_w) || !aligned16(down_w) || reinterpret_cast<uintptr_t>(packed) % 256 != 0)
    return fail(MOE_ERR_ALIGNMENT, "weights must be 16-byte and packed 256-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* P = static_cast<uint8_t*>(packed);
  const uint8_t* g = static_cast<const uint8_t*>(gate_w);
  const uint8_t* u = static_cast<const uint8_t*>(up_w);
  const size_t half_bytes = static_cast<size_t>(I) * H * 2;  // one expert's gate (or up) rows, 16-bit
  if (!q) {
    for (int64_t e = 0; e < E; ++e) {
      MOE_CUDA(cudaMemcpyAsync(P + off[0] + 2 * e * half_bytes, g + e * half_bytes, half_bytes,
                               cudaMemcpyDeviceToDevice, s));
      MOE_CUDA(cudaMemcpyAsync(P + off[0] + (2 * e + 1) * half_bytes, u + e * half_bytes, half_bytes,
                               cudaMemcpyDeviceToDevice, s));
    }
    MOE_CUDA(cudaMemcpyAsync(P + off[2], down_w, static_cast<size_t>(E) * H * I * 2, cudaMemcpyDeviceToDevice, s));
    return MOE_OK;
  }
  // per-row quantisation straight into the packed rows: expert e's gate rows land at rows
  // e * 2I .. e * 2I + I - 1 of w13, its up rows right after
  const bool fp8 = kind == MOE_F8E4M3;
  float* s13 = reinterpret_cast<float*>(P + off[1]);
  for (int64_t e = 0; e < E; ++e) {
    MOE_TRY(quantize_rows(fp8, g + e * half_bytes, dtype, I, H, P + off[0] + static_cast<size_t>(2 * e) * I * H,
                          s13 + 2 * e * I, stream));
    MOE_TRY(quantize_rows(fp8, u + e * half_bytes, dtype, I, H, P + off[0] + static_cast<size_t>(2 * e + 1) * I * H,
                          s13 + (2 * e + 1) * I, stream));
  }
  return quantize_rows(fp8, down_w, dtype, E * H, I, P + off[2], reinterpret_cast<float*>(P + off[3]), stream);
}

size_t moe_fused_packed_workspace_bytes(int64_t T, int64_t topk, int64_t E, int64_t H, int64_t I, int kind,
                                        int dtype) {
  if (kind == MOE_I8) return moe_fused_int8_workspace_bytes(T, topk, E, H, I, dtype);
  if (kind == MOE_F8E4M3) return moe_fused_fp8_workspace_bytes(T, topk, E, H, I, dtype);
  return moe_fused_workspace_bytes(T, topk, E, H, I, dtype);
}

int moe_fused_packed(const void* x, const void* packed, int kind, const void* ids, int ids_dtype, const void* tw,
                     int w_dtype, void* out, int64_t T, int64_t H, int64_t I, int64_t E, int64_t topk, int dtype,
                     void* workspace, size_t workspace_bytes, void* stream) {
  size_t off[4], total;
  MOE_TRY(moe_packed_weights_layout(E, H, I, kind, off, &total));
  if (!packed) return fail(MOE_ERR_INVALID_ARG, "null packed weights");
  const uint8_t* P = static_cast<const uint8_t*>(packed);
  const float* s13 = reinterpret_cast<const float*>(P + off[1]);
  const float* s2 = reinterpret_cast<const float*>(P + off[3]);
  if (kind == MOE_I8)
    return moe_fused_int8(x, P + off[0], s13, P + off[2], s2, ids, ids_dtype, tw, w_dtype, out, T, H, I, E, topk,
                          dtype, workspace, workspace_bytes, stream);
  if (kind == MOE_F8E4M3)
    return moe_fused_fp8(x, P + off[0], s13, P + off[2], s2, ids, ids_dtype, tw, w_dtype, out, T, H, I, E, topk,
                         dtype, workspace, workspace_bytes, stream);
  if (kind != dtype) return fail(MOE_ERR_INVALID_ARG, "16-bit packed weights must have the activation dtype");
  return moe_fused(x, P + off[0], P + off[2], ids, ids_dtype, tw, w_dtype, out, T, H, I, E, topk, dtype, workspace,
                   workspace_bytes, stream);
}

// ---------------------------------------------------------------------------- expert parallel
size_t moe_ep_plan_workspace_bytes(int64_t T, int64_t W) {
  if (T <= 0 || W <= 0) return 256;
  return round_up(sizeof(int32_t) * static_cast<size_t>(T * W), 256) + round_up(sizeof(int32_t) * (W + 1), 256) +
         moe_align_workspace_bytes(T * W, W);
}

int moe_ep_plan(const void* ids, int ids_dtype, int64_t T, int64_t topk, const int32_t* expert_rank, int64_t E,
                int64_t W, int32_t* send_counts, int32_t* send_offsets, int32_t* send_pairs, int32_t* pair_slot,
                int32_t* meta, void* workspace, size_t workspace_bytes, void* stream) {
  t_last_error.clear();
  if (W < 1 || W > kAlignMaxExperts) return fail(MOE_ERR_INVALID_ARG, "world must be in [1, %d]", kAlignMaxExperts);
  if (T < 0 || topk < 1 || E < 1) return fail(MOE_ERR_INVALID_ARG, "bad token/topk/expert count");
  if (T * W > (int64_t(1) << 31) - 1) return fail(MOE_ERR_INVALID_ARG, "num_tokens * world exceeds int32");
  if (ids_dtype != MOE_I32 && ids_dtype != MOE_I64) return fail(MOE_ERR_INVALID_ARG, "topk_ids must be int32 or int64");
  if (!send_counts || !send_offsets || !meta || (T > 0 && (!ids || !expert_rank || !send_pairs || !pair_slot)))
    return fail(MOE_ERR_INVALID_ARG, "null argument");
  if (!workspace || workspace_bytes < moe_ep_plan_workspace_bytes(T, W))
    return fail(MOE_ERR_WORKSPACE, "workspace must hold %zu bytes", moe_ep_plan_workspace_bytes(T, W));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* keys = reinterpret_cast<int32_t*>(ws);
  int32_t* padded = reinterpret_cast<int32_t*>(ws + round_up(sizeof(int32_t) * static_cast<size_t>(T * W), 256));
  int* counts = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(padded) + round_up(sizeof(int32_t) * (W + 1), 256));
  if (T > 0) {
    const int threads = 256;
    const int64_t n = T * W;
    const int blocks = static_cast<int>((n + threads - 1) / threads < 4096 ? (n + threads - 1) / threads : 4096);
    if (ids_dtype == MOE_I32)
      ep_pair_keys_kernel<int32_t><<<blocks, threads, 0, s>>>(static_cast<const int32_t*>(ids), (int)T, (int)topk,
                                                              expert_rank, (int)E, (int)W, keys);
    else
      ep_pair_keys_kernel<int64_t><<<blocks, threads, 0, s>>>(static_cast<const int64_t*>(ids), (int)T, (int)topk,
                                                              expert_rank, (int)E, (int)W, keys);
    MOE_CUDA(cudaGetLastError());
  }
  // block size 1: padded offsets equal the plain offsets; no block map
  MOE_TRY(launch_align(keys, MOE_I32, T * W, W, 1, send_counts, send_offsets, padded, nullptr, send_pairs, pair_slot,
                       meta, counts, s));
  return MOE_OK;
}

int moe_ep_pack(const void* x, const void* ids, int ids_dtype, const void* tw, int w_dtype, const int32_t* expert_rank,
                const int32_t* expert_local, int64_t E, const int32_t* send_pairs, const int32_t* meta, int64_t T,
                int64_t H, int64_t topk, int64_t W, int dtype, void* send_x, int32_t* send_ids, float* send_w,
                void* stream) {
  t_last_error.clear();
  if (dtype != MOE_F16 && dtype != MOE_BF16) return fail(MOE_ERR_INVALID_ARG, "dtype must be MOE_F16 or MOE_BF16");
  if (H <= 0 || H % 8 != 0) return fail(MOE_ERR_INVALID_ARG, "hidden must be a positive multiple of 8");
  if (ids_dtype != MOE_I32 && ids_dtype != MOE_I64) return fail(MOE_ERR_INVALID_ARG, "topk_ids must be int32 or int64");
  if (w_dtype != MOE_F32 && w_dtype != MOE_F16 && w_dtype != MOE_BF16)
    return fail(MOE_ERR_INVALID_ARG, "topk_weights must be fp32, fp16 or bf16");
  if (T == 0) return MOE_OK;
  if (!x || !ids || !tw || !expert_rank || !expert_local || !send_pairs || !meta || !send_x || !send_ids || !send_w)
    return fail(MOE_ERR_INVALID_ARG, "null argument");
  if (!aligned16(x) || !aligned16(send_x)) return fail(MOE_ERR_ALIGNMENT, "rows must be 16-byte aligned");
  int dev, sms;
  MOE_TRY(current_device(&dev));
  MOE_TRY(device_sms(dev, &sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int wd = w_dtype == MOE_F32 ? 0 : (w_dtype == MOE_F16 ? 1 : 2);
#define MOE_EP_PACK(TT, IT)                                                                                       \
  ep_pack_kernel<TT, IT><<<sms * 4, 256, 0, s>>>(static_cast<const TT*>(x), static_cast<const IT*>(ids), tw, wd,  \
                                                 expert_rank, expert_local, (int)E, send_pairs, meta, (int)H,     \
                                                 (int)topk, (int)W, static_cast<TT*>(send_x), send_ids, send_w)
  if (dtype == MOE_F16) {
    if (ids_dtype == MOE_I32) MOE_EP_PACK(__half, int32_t); else MOE_EP_PACK(__half, int64_t);
  } else {
    if (ids_dtype == MOE_I32) MOE_EP_PACK(__nv_bfloat16, int32_t); else MOE_EP_PACK(__nv_bfloat16, int64_t);
  }
#undef MOE_EP_PACK
  MOE_CUDA(cudaGetLastError());
  return MOE_OK;
}

int moe_ep_combine(const void* y, const int32_t* pair_slot, int64_t T, int64_t H, int64_t W, int dtype, void* out,
                   void* stream) {
  t_last_error.clear();
  if (dtype != MOE_F16 && dtype != MOE_BF16) return fail(MOE_ERR_INVALID_ARG, "dtype must be MOE_F16 or MOE_BF16");
  if (H <= 0 || H % 8 != 0 || W < 1) return fail(MOE_ERR_INVALID_ARG, "bad hidden or world");
  if (T == 0) return MOE_OK;
  if (!pair_slot || !out) return fail(MOE_ERR_INVALID_ARG, "null argument");
  int dev, sms;
  MOE_TRY(current_device(&dev));
  MOE_TRY(device_sms(dev, &sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == MOE_F16)
    ep_combine_kernel<__half><<<sms * 8, 256, 0, s>>>(static_cast<const __half*>(y), pair_slot, (int)T, (int)H, (int)W,
                                                      static_cast<__half*>(out));
  else
    ep_combine_kernel<__nv_bfloat16><<<sms * 8, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(y), pair_slot, (int)T,
                                                             (int)H, (int)W, static_cast<__nv_bfloat16*>(out));
  MOE_CUDA(cudaGetLastError());
  return MOE_OK;
}

// ---------------------------------------------------------------------------- EP over peer memory
static int ep_p2p_check(int64_t T_max, int64_t H, int64_t topk, int64_t W) {
  if (T_max < 1 || H < 8 || H % 8 != 0 || topk < 1 || W < 1 || W > 32)
    return fail(MOE_ERR_INVALID_ARG, "need max_tokens >= 1, hidden a multiple of 8, topk >= 1, 1 <= world <= 32");
  if (W * T_max * topk > (int64_t(1) << 31) - 1 || W * T_max > (int64_t(1) << 30))
    return fail(MOE_ERR_INVALID_ARG, "world * max_tokens * topk exceeds 32-bit indexing");
  return MOE_OK;
}

size_t moe_ep_region_bytes(int64_t T_max, int64_t H, int64_t topk, int64_t W) {
  if (T_max < 1 || H < 8 || topk < 1 || W < 1 || W > 32) return 0;
  return static_cast<size_t>(ep_region_layout(T_max, H, topk, W).total);
}

int moe_ep_region_alloc(size_t bytes, void** region) {
  t_last_error.clear();
  if (!region || bytes == 0) return fail(MOE_ERR_INVALID_ARG, "null region pointer or zero size");
  *region = nullptr;
  MOE_CUDA(cudaMalloc(region, bytes));
  MOE_CUDA(cudaMemset(*region, 0, bytes));
  return MOE_OK;
}

int moe_ep_region_free(void* region) {
  t_last_error.clear();
  if (region) MOE_CUDA(cudaFree(region));
  return MOE_OK;
}

int moe_ep_ipc_get(const void* region, void* handle) {
  t_last_error.clear();
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  if (!region || !handle) return fail(MOE_ERR_INVALID_ARG, "null argument");
  MOE_CUDA(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), const_cast<void*>(region)));
  return MOE_OK;
}

int moe_ep_ipc_open(const void* handle, void** region) {
  t_last_error.clear();
  if (!region || !handle) return fail(MOE_ERR_INVALID_ARG, "null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  MOE_CUDA(cudaIpcOpenMemHandle(region, h, cudaIpcMemLazyEnablePeerAccess));
  return MOE_OK;
}

int moe_ep_ipc_close(void* region) {
  t_last_error.clear();
  if (region) MOE_CUDA(cudaIpcCloseMemHandle(region));
  return MOE_OK;
}

int moe_ep_p2p_stage(void* region, const void* x, const void* ids, int ids_dtype, const void* tw, int w_dtype, int64_t T,
                     int64_t T_max, int64_t H, int64_t topk, int64_t W, int dtype, void* stream) {
  t_last_error.clear();
  MOE_TRY(ep_p2p_check(T_max, H, topk, W));
  if (dtype != MOE_F16 && dtype != MOE_BF16) return fail(MOE_ERR_INVALID_ARG, "dtype must be MOE_F16 or MOE_BF16");
  if (ids_dtype != MOE_I32 && ids_dtype != MOE_I64) return fail(MOE_ERR_INVALID_ARG, "topk_ids must be int32 or int64");
  if (w_dtype != MOE_F32 && w_dtype != MOE_F16 && w_dtype != MOE_BF16)
    return fail(MOE_ERR_INVALID_ARG, "topk_weights must be fp32, fp16 or bf16");
  if (T < 0 || T > T_max) return fail(MOE_ERR_INVALID_ARG, "num_tokens must be in [0, max_tokens]");
  if (!region || (T > 0 && (!x || !ids || !tw))) return fail(MOE_ERR_INVALID_ARG, "null argument");
  if (T > 0 && !aligned16(x)) return fail(MOE_ERR_ALIGNMENT, "hidden_states must be 16-byte aligned");
  int dev, sms;
  MOE_TRY(current_device(&dev));
  MOE_TRY(device_sms(dev, &sms));
  const EpRegion L = ep_region_layout(T_max, H, topk, W);
  const int wd = w_dtype == MOE_F32 ? 0 : (w_dtype == MOE_F16 ? 1 : 2);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* rg = static_cast<uint8_t*>(region);
  // one element type suffices for the row copy (16-byte vectors)
  if (ids_dtype == MOE_I32)
    ep_stage_kernel<__half, int32_t><<<sms * 4, 256, 0, s>>>(rg, L, static_cast<const __half*>(x),
                                                            static_cast<const int32_t*>(ids), tw, wd, (int)T, (int)H,
                                                            (int)topk);
  else
    ep_stage_kernel<__half, int64_t><<<sms * 4, 256, 0, s>>>(rg, L, static_cast<const __half*>(x),
                                                            static_cast<const int64_t*>(ids), tw, wd, (int)T, (int)H,
                                                            (int)topk);
  MOE_CUDA(cudaGetLastError());
  return MOE_OK;
}

int moe_ep_p2p_barrier(const uint64_t* regions, int rank, int W, uint32_t epoch, void* stream) {
  t_last_error.clear();
  if (!regions || W < 1 || W > 32 || rank < 0 || rank >= W) return fail(MOE_ERR_INVALID_ARG, "bad regions/rank/world");
  int dev;
  MOE_TRY(current_device(&dev));
  uint32_t* status;
  MOE_TRY(device_status_ptr(dev, &status));
  ep_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(regions, 0, rank, W, epoch, status);
  MOE_CUDA(cudaGetLastError());
  return MOE_OK;
}

static size_t ep_p2p_extra_bytes(int64_t T_max, int64_t topk, int64_t W) {
  return 2 * round_up(sizeof(int32_t) * static_cast<size_t>(W * T_max * topk), 256);
}

size_t moe_ep_p2p_workspace_bytes(int64_t T_max, int64_t topk, int64_t W, int64_t E_local, int64_t H, int64_t I,
                                  int dtype) {
  (void)dtype;
  if (T_max < 1 || topk < 1 || W < 1 || W > 32 || E_local < 1 || H < 1 || I < 1) return 0;
  return fused_layout(W * T_max, topk, E_local, H, I, false, false).total + ep_p2p_extra_bytes(T_max, topk, W);
}

static int ep_p2p_compute(bool push, const uint64_t* regions, void* own_region, int rank, int W, int64_t T_max,
                          int64_t H, int64_t I, int64_t topk, const int32_t* expert_rank, const int32_t* expert_local,
                          int64_t E, const void* w13, const void* w2, int64_t E_local, int dtype, void* workspace,
                          size_t workspace_bytes, void* stream) {
  t_last_error.clear();
  MOE_TRY(ep_p2p_check(T_max, H, topk, W));
  if (!regions || !own_region || rank < 0 || rank >= W || !expert_rank || !expert_local || E < 1 || E_local < 1)
    return fail(MOE_ERR_INVALID_ARG, "bad regions/rank/expert tables");
  if (push && topk > 32) return fail(MOE_ERR_UNSUPPORTED, "the push combine supports topk <= 32");
  const size_t need = moe_ep_p2p_workspace_bytes(T_max, topk, W, E_local, H, I, dtype);
  if (!workspace || workspace_bytes < need) return fail(MOE_ERR_WORKSPACE, "workspace must hold %zu bytes", need);
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return fail(MOE_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  int dev, sms;
  MOE_TRY(current_device(&dev));
  MOE_TRY(device_sms(dev, &sms));
  const EpRegion L = ep_region_layout(T_max, H, topk, W);
  uint8_t* extra = static_cast<uint8_t*>(workspace) + (need - ep_p2p_extra_bytes(T_max, topk, W));
  int32_t* local_ids = reinterpret_cast<int32_t*>(extra);
  float* local_w = reinterpret_cast<float*>(extra + ep_p2p_extra_bytes(T_max, topk, W) / 2);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ep_p2p_route_kernel<<<sms * 4, 256, 0, s>>>(regions, L, W, (int)T_max, (int)topk, expert_rank, expert_local, (int)E,
                                              rank, local_ids, local_w);
  MOE_CUDA(cudaGetLastError());
  PeerSource peer{regions, L, rank, W, (int)T_max, push};
  void* y = static_cast<uint8_t*>(own_region) + L.y;
  return fused_common(false, own_region, w13, nullptr, w2, nullptr, local_ids, MOE_I32,
                      local_w, MOE_F32, y, W * T_max, H, I, E_local, topk, dtype, workspace,
                      need - ep_p2p_extra_bytes(T_max, topk, W), stream, &peer);
}

int moe_ep_p2p_compute(const uint64_t* regions, void* own_region, int rank, int W, int64_t T_max, int64_t H, int64_t I,
                       int64_t topk, const int32_t* expert_rank, const int32_t* expert_local, int64_t E,
                       const void* w13, const void* w2, int64_t E_local, int dtype, void* workspace,
                       size_t workspace_bytes, void* stream) {
  return ep_p2p_compute(false, regions, own_region, rank, W, T_max, H, I, topk, expert_rank, expert_local, E, w13, w2,
                        E_local, dtype, workspace, workspace_bytes, stream);
}

int moe_ep_p2p_compute_push(const uint64_t* regions, void* own_region, int rank, int W, int64_t T_max, int64_t H,
                            int64_t I, int64_t topk, const int32_t* expert_rank, const int32_t* expert_local,
                            int64_t E, const void* w13, const void* w2, int64_t E_local, int dtype, void* workspace,
                            size_t workspace_bytes, void* stream) {
  return ep_p2p_compute(true, regions, own_region, rank, W, T_max, H, I, topk, expert_rank, expert_local, E, w13, w2,
                        E_local, dtype, workspace, workspace_bytes, stream);
}

// Push combine, home side: nothing to prepare (every slot a forward reads is written by its owner
// in that forward); after the second barrier, sum each own token's slots into out.
int moe_ep_p2p_push_prepare(void* own_region, int64_t T, int64_t T_max, int64_t H, int64_t topk, int W, int dtype,
                            void* stream) {
  t_last_error.clear();
  (void)stream;
  MOE_TRY(ep_p2p_check(T_max, H, topk, W));
  if (dtype != MOE_F16 && dtype != MOE_BF16) return fail(MOE_ERR_INVALID_ARG, "dtype must be MOE_F16 or MOE_BF16");
  if (T < 0 || T > T_max) return fail(MOE_ERR_INVALID_ARG, "num_tokens must be in [0, max_tokens]");
  if (!own_region) return fail(MOE_ERR_INVALID_ARG, "null region");
  return MOE_OK;
}

int moe_ep_p2p_push_finish(const void* own_region, int64_t T, int64_t T_max, int64_t H, int64_t topk, int W, int64_t E,
                           int dtype, void* out, void* stream) {
  t_last_error.clear();
  MOE_TRY(ep_p2p_check(T_max, H, topk, W));
  if (dtype != MOE_F16 && dtype != MOE_BF16) return fail(MOE_ERR_INVALID_ARG, "dtype must be MOE_F16 or MOE_BF16");
  if (T < 0 || T > T_max) return fail(MOE_ERR_INVALID_ARG, "num_tokens must be in [0, max_tokens]");
  if (E < 1 || E > (int64_t(1) << 30)) return fail(MOE_ERR_INVALID_ARG, "num_experts out of range");
  if (topk > 32) return fail(MOE_ERR_UNSUPPORTED, "the push combine supports topk <= 32");
  if (T == 0) return MOE_OK;
  if (!own_region || !out) return fail(MOE_ERR_INVALID_ARG, "null argument");
  if (!aligned16(out)) return fail(MOE_ERR_ALIGNMENT, "out must be 16-byte aligned");
  int dev, sms;
  MOE_TRY(current_device(&dev));
  MOE_TRY(device_sms(dev, &sms));
  const EpRegion L = ep_region_layout(T_max, H, topk, W);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* region = static_cast<const uint8_t*>(own_region);
  if (dtype == MOE_F16)
    ep_push_combine_kernel<__half><<<sms * 8, 256, 0, s>>>(region, L, (int)T, (int)H, (int)topk, (int)E,
                                                           static_cast<__half*>(out));
  else
    ep_push_combine_kernel<__nv_bfloat16><<<sms * 8, 256, 0, s>>>(region, L, (int)T, (int)H, (int)topk, (int)E,
                                                                  static_cast<__nv_bfloat16*>(out));
  MOE_CUDA(cudaGetLastError());
  return MOE_OK;
}

int moe_ep_p2p_combine(const uint64_t* regions, int rank, int W, int64_t T, int64_t T_max, int64_t H, int64_t topk,
                       const int32_t* expert_rank, int64_t E, int dtype, void* out, void* stream) {
  t_last_error.clear();
  MOE_TRY(ep_p2p_check(T_max, H, topk, W));
  if (dtype != MOE_F16 && dtype != MOE_BF16) return fail(MOE_ERR_INVALID_ARG, "dtype must be MOE_F16 or MOE_BF16");
  if (T < 0 || T > T_max) return fail(MOE_ERR_INVALID_ARG, "num_tokens must be in [0, max_tokens]");
  if (T == 0) return MOE_OK;
  if (!regions || rank < 0 || rank >= W || !expert_rank || !out) return fail(MOE_ERR_INVALID_ARG, "null argument");
  if (!aligned16(out)) return fail(MOE_ERR_ALIGNMENT, "out must be 16-byte aligned");
  int dev, sms;
  MOE_TRY(current_device(&dev));
  MOE_TRY(device_sms(dev, &sms));
  const EpRegion L = ep_region_layout(T_max, H, topk, W);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == MOE_F16)
    ep_combine_pull_kernel<__half><<<sms * 8, 256, 0, s>>>(regions, L, rank, W, (int)T_max, (int)T, (int)H, (int)topk,
                                                           expert_rank, (int)E, static_cast<__half*>(out));
  else
    ep_combine_pull_kernel<__nv_bfloat16><<<sms * 8, 256, 0, s>>>(regions, L, rank, W, (int)T_max, (int)T, (int)H,
                                                                  (int)topk, expert_rank, (int)E,
                                                                  static_cast<__nv_bfloat16*>(out));
  MOE_CUDA(cudaGetLastError());
  return MOE_OK;
}

}  // extern "C"
