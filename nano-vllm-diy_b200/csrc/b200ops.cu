// C-ABI of the B200 decoder-path kernels (libb200ops.so).
//
// Every entry point takes raw device pointers, sizes and a cudaStream_t,
// allocates nothing, launches on the given stream (so it can be captured in a
// CUDA graph) and returns B200_OK or a negative status.  The message of the
// last failure on the calling thread is available from b200_last_error().
// Declarations and the reference interface each one replaces are in
// include/b200ops.h.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "attention.cuh"
#include "decode_attention.cuh"
#include "common.cuh"
#include "elementwise.cuh"
#include "exchange.cuh"
#include "metadata.cuh"
#include "prefill_tc.cuh"
#include "gemm.cuh"
#include "gemm_pair.cuh"
#include "../../include/b200ops.h"

using namespace b200;

namespace {

thread_local std::string g_last_error;

// Guards the host-side per-device state and lookup caches below (filled on
// first use; several host threads may drive the library).  Taken only in
// leaf functions, which never call one another while holding it.
std::mutex g_host_mutex;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

// Number of kernels this library has launched from the host (graph replays
// launch without the host and are not counted).
unsigned long long g_launches = 0;

int check_launch(const char* what) {
  ++g_launches;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return B200_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Programmatic dependent launch of the kernels of this library (each one
// waits for its predecessor with griddepcontrol.wait before it reads its
// inputs, a no-op under a plain launch).  Off unless B200_PDL=1 (every
// kernel) or B200_PDL=gemm (the GEMM kernels only): measured on the Qwen3-8B
// decode step, on every kernel it gained nothing at tp 1 and cost 4.5 % at
// tp 2 (early-launched dependents take SM resources from the running kernel).
bool pdl_enabled(bool gemm = false) {
  const char* e = getenv("B200_PDL");
  if (!e) return false;
  if (*e == '1') return true;
  return gemm && std::strcmp(e, "gemm") == 0;
}

// cudaLaunchKernelEx with the given attributes plus programmatic stream
// serialization.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                      const cudaLaunchAttribute* extra, int nextra, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[4];
  int n = 0;
  for (int i = 0; i < nextra && n < 3; ++i) attr[n++] = extra[i];
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

constexpr int kMaxDevices = 64;

// Per-device state: SM count, the device error word's address and which
// kernels already had their dynamic shared memory limit raised.
struct DeviceState {
  bool init = false;
  int num_sms = 0;
  unsigned* err = nullptr;
  unsigned smem_configured = 0;
};
DeviceState g_dev[kMaxDevices];

__device__ unsigned g_device_error_word;

int device_state(DeviceState** out) {
  std::lock_guard<std::mutex> lock(g_host_mutex);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(B200_ERR_INVALID, "device %d out of range", dev);
  DeviceState& s = g_dev[dev];
  if (!s.init) {
    e = cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(B200_ERR_CUDA, "SM count: %s", cudaGetErrorString(e));
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_device_error_word);
    if (e != cudaSuccess) return fail(B200_ERR_CUDA, "error word: %s", cudaGetErrorString(e));
    s.err = static_cast<unsigned*>(p);
    s.init = true;
  }
  *out = &s;
  return B200_OK;
}

// Raise a kernel's dynamic shared-memory limit to at least `bytes` (once per
// kernel, device and size; the limit must leave room for static smem).
template <typename K>
int ensure_smem(DeviceState* ds, unsigned bit, K kernel, int bytes) {
  static int configured[kMaxDevices][8] = {};
  std::lock_guard<std::mutex> lock(g_host_mutex);
  int dev = 0;
  cudaGetDevice(&dev);
  int slot = 0;
  while ((1u << slot) != bit && slot < 7) ++slot;
  if (configured[dev][slot] >= bytes) return B200_OK;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "smem attribute (%d bytes): %s", bytes, cudaGetErrorString(e));
  configured[dev][slot] = bytes;
  (void)ds;
  return B200_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::lock_guard<std::mutex> lock(g_host_mutex);
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  std::lock_guard<std::mutex> lock(g_host_mutex);
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 3020, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  }
  return fn;
}

// 2-D bf16 tensor map with the given swizzle (zero fill outside on loads,
// clipping on stores).
int make_tmap_sw(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows,
                 uint64_t row_stride, uint32_t box_inner, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride * 2};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                         CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return B200_OK;
}

// 2-D bf16 tensor map: `rows` rows of `inner` elements, `row_stride` elements
// apart, box = box_inner x box_rows, 128-byte swizzle, zero fill outside.
int make_tmap(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows,
              uint64_t row_stride, uint32_t box_inner, uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride * 2};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return B200_OK;
}

// 3-D bf16 tensor map: dims {d0 (contiguous), d1, d2} with byte strides
// {s1, s2} for d1 / d2, box {b0, b1, b2}, 128-byte swizzle, zero fill outside.
int make_tmap_3d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t s1_bytes, uint64_t s2_bytes, uint32_t b0, uint32_t b1, uint32_t b2) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1_bytes, s2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
  return B200_OK;
}

// ---------------------------------------------------------------------------
// GEMM planning
// ---------------------------------------------------------------------------
struct GemmPlan {
  int BN, token_tiles, n_tiles, num_kb, kb_per_split, splits, stages, smem, tmem_cols;
  int kstep = 1;  // SM-pair kernel: 64-wide K blocks per ring stage
  // SM-pair kernel schedule (GemmArgs::sched, grp_*, csplit)
  int sched, grp_whole, grp_split, grp_size, csplit;
};

int round_up(int x, int m) { return (x + m - 1) / m * m; }

// Two CTAs per SM: each CTA's ring stays under ~110 KB, so the epilogue of
// one CTA overlaps the main loop of the other.
constexpr int kGemmSmemBudget = 110 * 1024;

bool gemm_debug() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("B200_GEMM_DEBUG");
    v = (e && *e && *e != '0') ? 1 : 0;
  }
  return v == 1;
}

// Optional override "BN,S,budget_kb" from B200_GEMM_CONFIG (tuning sweeps).
bool gemm_forced(int* bn, int* s, int* budget) {
  const char* e = getenv("B200_GEMM_CONFIG");
  if (!e || !*e) return false;
  return sscanf(e, "%d,%d,%d", bn, s, budget) == 3;
}

GemmPlan plan_gemm(DeviceState* ds, int T, int N, int K, bool silu_tiles) {
  GemmPlan p{};
  int f_bn = 0, f_s = 0, f_budget = 0;
  const bool forced = gemm_forced(&f_bn, &f_s, &f_budget);
  p.BN = std::min(128, std::max(32, round_up(T, 32)));
  if (forced) p.BN = std::min(256, std::max(32, std::min(f_bn, round_up(T, 32))));
  p.token_tiles = (T + p.BN - 1) / p.BN;
  p.n_tiles = silu_tiles ? (N / 2 + 63) / 64 : (N + kGemmBM - 1) / kGemmBM;
  p.num_kb = (K + kGemmBK - 1) / kGemmBK;
  const int stage = kGemmBM * kGemmBK * 2 + p.BN * kGemmBK * 2;
  const int budget = forced ? f_budget * 1024 : kGemmSmemBudget;
  p.stages = std::max(2, std::min(kGemmMaxStages, (budget - 2048) / stage));
  while (p.stages * stage < p.BN * kGemmBM * 4) ++p.stages;  // ring holds the fp32 tile
  p.smem = 1024 + p.stages * stage + 256;
  p.tmem_cols = 32;
  while (p.tmem_cols < p.BN) p.tmem_cols <<= 1;
  // split K over a cluster when the tiles leave SMs idle: measured on the
  // Qwen3-8B decode shapes (T = 256), 2-way splits win for K <= 8192 and
  // 4-way for longer K; every rank keeps >= 8 K blocks
  const int tiles = p.n_tiles * p.token_tiles;
  int best_s = 1;
  if (tiles < ds->num_sms) best_s = p.num_kb >= 128 ? 4 : 2;
  while (best_s > 1 && p.num_kb / best_s < 8) --best_s;
  if (gemm_debug())
    fprintf(stderr, "[b200 gemm] T=%d N=%d K=%d BN=%d tiles=%d S=%d\n", T, N, K, p.BN, tiles, best_s);
  if (forced) best_s = std::max(1, std::min(8, std::min(f_s, p.num_kb)));
  p.kb_per_split = (p.num_kb + best_s - 1) / best_s;
  p.splits = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;
  if (gemm_debug())
    fprintf(stderr, "[b200 gemm] -> T=%d N=%d K=%d BN=%d tiles=%d splits=%d stages=%d smem=%d\n", T, N,
            K, p.BN, tiles, p.splits, p.stages, p.smem);
  return p;
}

// Decode attention: one CTA per SM, launched cooperatively (its merge phase
// follows a grid-wide barrier, so every CTA must be resident).
int launch_decode(DeviceState* ds, const CUtensorMap& tmK, const CUtensorMap& tmV,
                  const CUtensorMap& tmQ, const DecodeArgs& a, int smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ds->num_sms, 1, 1);
  cfg.blockDim = dim3(kDecWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_attn_kernel, tmK, tmV, tmQ, a);
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "decode attention launch: %s", cudaGetErrorString(e));
  return B200_OK;
}

// ---------------------------------------------------------------------------
// SM-pair GEMM (gemm_pair_tcgen05_kernel): one CTA per SM, clusters of 2
// ---------------------------------------------------------------------------
constexpr int kPairSmemBudget = 226 * 1024;  // one CTA per SM (227 KB opt-in limit)

// B200_GEMM_PAIR=0 selects the single-SM kernel for every shape and
// B200_GEMM_PAIR=2 the SM-pair kernel for every shape; B200_GEMM_SCHED=
// streamk keeps the SM-pair kernel on its stream-K schedule.  Read at every
// call, so a process can compare the kernels and schedules.
bool pair_enabled() {
  const char* e = getenv("B200_GEMM_PAIR");
  return !(e && *e == '0');
}
bool pair_forced() {
  const char* e = getenv("B200_GEMM_PAIR");
  return e && *e == '2';
}
// B200_GEMM_PAIR=3: the SM-pair kernel's cluster split-K mode for plain
// (non-SiLU) GEMMs.
bool csk_forced() {
  const char* e = getenv("B200_GEMM_PAIR");
  return e && *e == '3';
}

bool grouped_allowed() {
  const char* e = getenv("B200_GEMM_SCHED");
  return !(e && std::strcmp(e, "streamk") == 0);
}

struct PairSchedule {
  int sched, pairs, whole, split, group;
};

// Work split of the SM-pair kernel over at most `max_pairs` co-resident
// pairs.  Grouped (sched 1) when every split tile gets a group of at least
// 2 pairs (or no tile is split): w = tiles / P whole tiles per pair, r =
// tiles % P split tiles shared by g = min(8, P / r, K blocks) pairs each.
// Otherwise stream-K (sched 0) over as many pairs as keep >= max(4, K
// blocks / 4) units each, so a stream-K tile has at most 5 sharers.
PairSchedule pair_schedule(long long tiles, int num_kb, int max_pairs, bool allow_grouped) {
  PairSchedule s{};
  max_pairs = std::max(1, max_pairs);
  const long long w = tiles / max_pairs, r = tiles % max_pairs;
  const long long g = r > 0 ? std::min<long long>(std::min<long long>(8, max_pairs / r), num_kb) : 0;
  if (allow_grouped && (r == 0 || g >= 2)) {
    s.sched = 1;
    s.whole = (int)w;
    s.split = (int)r;
    s.group = (int)g;
    s.pairs = w > 0 ? max_pairs : (int)(r * g);
    return s;
  }
  const long long total = tiles * num_kb;
  const long long min_units = std::max(4, (num_kb + 3) / 4);
  s.sched = 0;
  s.pairs = (int)std::max(1LL, std::min<long long>(max_pairs, total / min_units));
  return s;
}

// Co-resident CTAs of the pair kernel with clusters of (2 x splits, 1, 1) and
// the given dynamic shared memory (occupancy queries are slow: cached).
long long pair_resident(int splits, int smem) {
  static long long cache[kMaxDevices][5][4] = {};
  static int cache_smem[kMaxDevices][5][4] = {};
  std::lock_guard<std::mutex> lock(g_host_mutex);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices || splits < 1 || splits > 4) return 0;
  for (int i = 0; i < 4; ++i)
    if (cache_smem[dev][splits][i] == smem) return cache[dev][splits][i];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * splits, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2 * splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, gemm_pair_tcgen05_kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    clusters = 0;
  }
  const long long v = (long long)clusters * 2 * splits;
  for (int i = 0; i < 4; ++i)
    if (cache_smem[dev][splits][i] == 0) {
      cache_smem[dev][splits][i] = smem;
      cache[dev][splits][i] = v;
      break;
    }
  return v;
}

// Workspace of the persistent pair kernel: 4 KiB of partial-ready flags,
// then one fp32 [256][128] partial tile per CTA (at most one CTA per SM).
size_t pair_workspace_bytes(int num_sms) { return 4096 + (size_t)num_sms * 256 * kGemmBM * 4; }

// Plan of the persistent SM-pair kernel: tokens in tiles of 256 (128 per
// CTA), BN = NP = the pair's weight rows per tile (<= 256; the gate_up
// projection always 256 = 128 gate + the 128 matching up rows), n_tiles =
// 2 x feature tiles, TMEM = two accumulators of pow2(NP) columns.
// `splits` holds the number of pairs launched (pair_schedule over the
// co-resident pairs).
// 64-wide K blocks per ring stage of the SM-pair kernel: 2 (one 32-64 KB
// stage per two blocks, half the barrier round trips per byte; measured
// faster TMA streaming with the same bytes in flight) unless B200_GEMM_KSTEP=1.
int pair_kstep() {
  const char* e = getenv("B200_GEMM_KSTEP");
  return (e && *e == '1') ? 1 : 2;
}

GemmPlan plan_pair(DeviceState* ds, int T, int N, int K, bool silu_tiles, int* rc) {
  GemmPlan p{};
  p.BN = silu_tiles ? 256 : std::min(256, std::max(32, round_up(N, 32)));
  p.token_tiles = (T + 2 * kGemmBM - 1) / (2 * kGemmBM);
  p.n_tiles = 2 * (silu_tiles ? (N / 2 + 127) / 128 : (N + p.BN - 1) / p.BN);
  p.num_kb = (K + kGemmBK - 1) / kGemmBK;
  p.kstep = pair_kstep();
  const int stage = p.kstep * (kGemmBM * kGemmBK * 2 + (p.BN / 2) * kGemmBK * 2);
  const int extra = 4 * kGemmBM * 64 + 512;  // output staging + barriers
  p.stages = std::min(kGemmMaxStages, (kPairSmemBudget - 1024 - extra) / stage);
  p.smem = 1024 + p.stages * stage + extra;
  int cols = 32;
  while (cols < p.BN) cols <<= 1;
  p.tmem_cols = 2 * cols;
  *rc = ensure_smem(ds, 8u, gemm_pair_tcgen05_kernel, p.smem);
  if (*rc) return p;
  const long long tiles = (long long)(p.n_tiles / 2) * p.token_tiles;
  long long max_pairs = pair_resident(1, p.smem) / 2;
  max_pairs = std::min(max_pairs, (long long)ds->num_sms / 2);
  const char* forced = getenv("B200_GEMM_PAIRS");
  if (forced && *forced) max_pairs = std::max(1LL, std::min(max_pairs, (long long)atoi(forced)));
  const PairSchedule sc = pair_schedule(tiles, p.num_kb, (int)std::max(1LL, max_pairs), grouped_allowed());
  p.sched = sc.sched;
  p.grp_whole = sc.whole;
  p.grp_split = sc.split;
  p.grp_size = sc.group;
  p.splits = sc.pairs;
  if (gemm_debug())
    fprintf(stderr,
            "[b200 gemm pair] T=%d N=%d K=%d NP=%d tiles=%dx%d kb=%d pairs=%d sched=%d whole=%d split=%d "
            "group=%d stages=%d smem=%d\n",
            T, N, K, p.BN, p.n_tiles / 2, p.token_tiles, p.num_kb, p.splits, p.sched, p.grp_whole,
            p.grp_split, p.grp_size, p.stages, p.smem);
  return p;
}

// Plan of the pair kernel's cluster split-K mode (plain GEMMs): clusters of C
// pairs (2C CTAs, C = 2..4), one tile each, K split C ways.  Among the (C, NP)
// whose clusters are all co-resident (NP a multiple of 32, <= 256, the ring
// able to receive the other members' partials), pick the smallest modelled
// time: per SM, the TMA ingest of its K share (128 token rows + NP/2 weight
// rows per 64-wide K block, ~74 GB/s measured per SM) plus the partial chunks
// it receives through distributed shared memory.  B200_GEMM_CSK="C,NP" forces
// a configuration (tuning).  `splits` = pairs launched (C per tile), 0 when
// the mode does not apply; *resident tells whether every cluster is resident.
GemmPlan plan_pair_cluster(DeviceState* ds, int T, int N, int K, bool* resident, int* rc) {
  GemmPlan best{};
  double best_cost = 1e300;
  *rc = 0;
  *resident = false;
  const int num_kb = (K + kGemmBK - 1) / kGemmBK;
  if (num_kb < 2) return best;
  int f_c = 0, f_np = 0;
  const char* fe = getenv("B200_GEMM_CSK");
  const bool forced = fe && *fe && sscanf(fe, "%d,%d", &f_c, &f_np) == 2;
  const int token_tiles = (T + 2 * kGemmBM - 1) / (2 * kGemmBM);
  for (int c = 2; c <= 4; ++c) {
    if (num_kb < c || (forced && c != f_c)) continue;
    for (int np = 32; np <= 256; np += 32) {
      if (forced && np != f_np) continue;
      GemmPlan p{};
      p.BN = np;
      p.token_tiles = token_tiles;
      p.n_tiles = 2 * ((N + np - 1) / np);
      p.num_kb = num_kb;
      p.kstep = pair_kstep();
      const int blk = kGemmBM * kGemmBK * 2 + (np / 2) * kGemmBK * 2;  // one 64-wide K block
      const int stage = p.kstep * blk;
      const int extra = 4 * kGemmBM * 64 + 512;
      p.stages = std::min(kGemmMaxStages, (kPairSmemBudget - 1024 - extra) / stage);
      p.smem = 1024 + p.stages * stage + extra;
      int cols = 32;
      while (cols < np) cols <<= 1;
      p.tmem_cols = 2 * cols;
      // the ring receives ceil(NP/32 / C) chunks from each of the C - 1 others
      const int nchunks = np / 32;
      const long long recv = (long long)((nchunks + c - 1) / c) * (c - 1) * kChunkFloats * 4;
      if ((long long)p.stages * stage < recv) continue;
      if ((*rc = ensure_smem(ds, 8u, gemm_pair_tcgen05_kernel, p.smem))) return GemmPlan{};
      const long long tiles = (long long)(p.n_tiles / 2) * token_tiles;
      const bool all_resident = tiles * 2 * c <= pair_resident(c, p.smem);
      if (!all_resident && !forced) continue;
      p.sched = 0;
      p.csplit = c;
      p.splits = (int)(c * tiles);
      const double kb_share = (double)((num_kb + c - 1) / c);
      const double cost = kb_share * (double)blk / 74e3 + (double)recv / 150e3 + 1.0;  // us
      if (cost < best_cost) {
        best_cost = cost;
        best = p;
        *resident = all_resident;
      }
    }
  }
  if (gemm_debug() && best.splits)
    fprintf(stderr, "[b200 gemm pair] T=%d N=%d K=%d NP=%d tiles=%d kb=%d cluster split-K C=%d pairs=%d smem=%d cost=%.1f\n",
            T, N, K, best.BN, best.n_tiles / 2 * best.token_tiles, best.num_kb, best.csplit, best.splits,
            best.smem, best_cost);
  return best;
}

int launch_pair(const GemmPlan& p, const CUtensorMap& tmW, const CUtensorMap& tmX,
                const CUtensorMap& tmY, const GemmArgs& a, cudaStream_t st, const char* what) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * p.splits, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.csplit >= 2 ? 2 * p.csplit : 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled(true) ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_pair_tcgen05_kernel, tmW, tmX, tmY, a);
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}

// RMSNorm (+ residual add) ahead of a GEMM: x (+ residual) normalised by
// weight into the GEMM's X operand (b200_rmsnorm_linear).
struct NormIn {
  const void* x;
  long long ldx;
  const void* residual;
  void* residual_out;
  const void* weight;
  float eps;
};

// RMSNorm (+ residual add) rows on rms_norm_kernel (b200_rms_norm).
int launch_rms_norm(const void* x, long long x_stride, const void* residual, const void* weight,
                    void* out, long long out_stride, void* residual_out, int rows, int dim, float eps,
                    cudaStream_t st) {
  if (rows <= 0) return B200_OK;
  if (dim <= 0 || dim % 8 || dim > 8 * 256 * 4)
    return fail(B200_ERR_UNSUPPORTED, "rms_norm: dim %d must be a multiple of 8 and <= 8192", dim);
  if (x_stride % 8 || out_stride % 8 || !aligned16(x) || !aligned16(out) || !aligned16(weight))
    return fail(B200_ERR_INVALID, "rms_norm: rows must be 16-byte aligned");
  if (residual && (!residual_out || !aligned16(residual) || !aligned16(residual_out)))
    return fail(B200_ERR_INVALID, "rms_norm: residual needs an aligned residual_out");
  const int nvec = dim / 8;
  const int threads = nvec >= 256 ? 256 : max(32, round_up(nvec, 32));
  const int vpt = (nvec + threads - 1) / threads;
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto R = static_cast<const __nv_bfloat16*>(residual);
  auto W = static_cast<const __nv_bfloat16*>(weight);
  auto O = static_cast<__nv_bfloat16*>(out);
  auto RO = static_cast<__nv_bfloat16*>(residual_out);
#define B200_LAUNCH_NORM(V)                                                                      \
  do {                                                                                           \
    if (residual)                                                                                \
      launch_ex(rms_norm_kernel<V, true>, dim3(rows), dim3(threads), 0, st, nullptr, 0, X,       \
                x_stride, R, W, O, out_stride, RO, dim, eps);                                    \
    else                                                                                         \
      launch_ex(rms_norm_kernel<V, false>, dim3(rows), dim3(threads), 0, st, nullptr, 0, X,      \
                x_stride, R, W, O, out_stride, RO, dim, eps);                                    \
  } while (0)
  if (vpt <= 1) B200_LAUNCH_NORM(1);
  else if (vpt <= 2) B200_LAUNCH_NORM(2);
  else B200_LAUNCH_NORM(4);
#undef B200_LAUNCH_NORM
  return check_launch("rms_norm_kernel");
}

// Word offset (in the pair workspace's flag area) of the fused RMSNorm's
// grid barrier: arrivals, generation.
constexpr int kNormBarrierWord = 1000;

// Whether an eligible GEMM takes its RMSNorm inside its own launch: only
// with B200_FUSE_NORM=1.  Measured slower in the Qwen3-8B decode step (21.7-
// 21.8k against 22.4-22.5k tok/s, same box): the norm rows on four warps per
// CTA plus the grid barrier take longer than the rms_norm launch they replace.
bool fuse_norm_enabled() {
  const char* e = getenv("B200_FUSE_NORM");
  return e && *e == '1';
}

int run_gemm(const void* x, long long ldx, const void* w, long long ldw, const void* bias, void* y,
             long long ldy, int T, int N, int K, bool silu, void* workspace, size_t ws_bytes,
             cudaStream_t st, const NormIn* norm = nullptr) {
  if (T <= 0) return B200_OK;
  if (N <= 0 || K <= 0) return fail(B200_ERR_INVALID, "linear: bad shape N=%d K=%d", N, K);
  if (K % 8 || ldx % 8 || ldw % 8 || ldx < K || ldw < K)
    return fail(B200_ERR_INVALID, "linear: K (%d) and row strides (%lld, %lld) must be multiples of 8", K, ldx, ldw);
  if (!aligned16(x) || !aligned16(w)) return fail(B200_ERR_INVALID, "linear: x and w must be 16-byte aligned");
  if (silu && (N % 2 || (N / 2) % 64 || ldy < N / 2))
    return fail(B200_ERR_UNSUPPORTED, "linear_silu: I = %d must be a multiple of 64", N / 2);
  if (!silu && ldy < N) return fail(B200_ERR_INVALID, "linear: ldy < N");
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  // Kernel choice: the SM-pair kernel when every pair gets at least one
  // whole tile (large projections such as gate_up and the LM head), where
  // the grouped schedule's split-K exchange overlaps the MMAs of the whole
  // tiles; otherwise the single-SM kernel with its on-chip cluster split-K
  // (measured faster for the smaller projections: with no whole tile to hide
  // it behind, the exchange through L2 costs more than it saves).
  const long long pair_tiles = (long long)(silu ? (N / 2 + 127) / 128 : (N + 255) / 256) *
                               ((T + 2 * kGemmBM - 1) / (2 * kGemmBM));
  const bool use_pair = pair_enabled() && workspace != nullptr && aligned16(workspace) &&
                        ws_bytes >= pair_workspace_bytes(ds->num_sms) &&
                        (pair_forced() || pair_tiles >= ds->num_sms / 2);
  // The pair kernel's cluster split-K mode also takes plain GEMMs with more
  // than 128 tokens and fewer tiles than pairs when its tiles stay at least
  // 192 rows wide with every cluster resident (measured: qkv 6144 x 4096 at
  // T = 256 22.8 us against 24.5; with 128-row tiles the token bytes each SM
  // reads outweigh the on-chip reduction: o_proj even, down 48.8 against 38.2).
  GemmPlan pp{};
  bool pair = use_pair;
  const bool csk_ok = !silu && pair_enabled() && workspace != nullptr && aligned16(workspace) &&
                      ws_bytes >= pair_workspace_bytes(ds->num_sms);
  bool csk_used = false;
  bool all_resident = true;  // every CTA of the pair launch co-resident
  if (csk_ok && (csk_forced() || (!use_pair && T > kGemmBM))) {
    int prc = 0;
    bool resident = false;
    const GemmPlan cp = plan_pair_cluster(ds, T, N, K, &resident, &prc);
    if (prc) return prc;
    // narrow projections (N <= 2048: qkv per rank at tp 4 / 8) take it whatever
    // the tile width: qkv 1536 x 4096 at T = 256 measured 14.6 us against 20.4
    // on the single-SM kernel, 768 x 4096 13.5 against 20.1
    if (cp.splits > 0 && (csk_forced() || (resident && (cp.BN >= 192 || N <= 2048)))) {
      pp = cp;
      pair = csk_used = true;
      all_resident = resident;
    }
  }
  // RMSNorm fused into the launch (a grid barrier between the rows and the
  // first activation loads) only on the persistent pair kernel with every CTA
  // resident; otherwise its own launch ahead of the GEMM
  const bool fuse = norm != nullptr && pair && all_resident && fuse_norm_enabled();
  if (norm != nullptr && !fuse) {
    if (int r = launch_rms_norm(norm->x, norm->ldx, norm->residual, norm->weight, const_cast<void*>(x), ldx,
                                norm->residual_out, T, K, norm->eps, st))
      return r;
  }
  if (!csk_used && use_pair) {
    int prc = 0;
    pp = plan_pair(ds, T, N, K, silu, &prc);
    if (prc) return prc;
  }
  if (pair) {
    const GemmPlan& p = pp;
    CUtensorMap tmW, tmX;
    if (int r = make_tmap(&tmW, w, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, kGemmBK,
                          (uint32_t)(p.BN / 2)))
      return r;
    if (int r = make_tmap(&tmX, x, (uint64_t)K, (uint64_t)T, (uint64_t)ldx, kGemmBK,
                          (uint32_t)kGemmBM))
      return r;
    GemmArgs a{};
    a.T = T; a.N = N; a.K = K; a.BN = p.BN; a.stages = p.stages; a.num_kb = p.num_kb;
    a.kb_per_split = p.kb_per_split; a.splits = p.splits; a.tmem_cols = p.tmem_cols;
    a.kstep = p.kstep;
    a.epi = silu ? EPI_SILU : EPI_BF16;
    a.vec_ok = aligned16(y) && (ldy % 8 == 0);
    a.y = static_cast<__nv_bfloat16*>(y); a.ldy = ldy;
    a.bias = static_cast<const __nv_bfloat16*>(bias);
    a.silu_inter = N / 2;
    a.tiles_m = p.n_tiles / 2;
    a.tiles_t = p.token_tiles;
    a.sk_flags = static_cast<unsigned*>(workspace);
    a.sk_part = reinterpret_cast<float*>(static_cast<char*>(workspace) + 4096);
    a.sched = p.sched;
    a.grp_whole = p.grp_whole;
    a.grp_split = p.grp_split;
    a.grp_size = p.grp_size;
    a.csplit = p.csplit;
    a.err = ds->err;
    if (fuse) {
      a.nx = static_cast<const __nv_bfloat16*>(norm->x);
      a.ldnx = norm->ldx;
      a.nres = static_cast<const __nv_bfloat16*>(norm->residual);
      a.nres_out = static_cast<__nv_bfloat16*>(norm->residual_out);
      a.nw = static_cast<const __nv_bfloat16*>(norm->weight);
      a.neps = norm->eps;
      a.nxo = static_cast<__nv_bfloat16*>(const_cast<void*>(x));
      a.ldnxo = ldx;
      a.gbar = static_cast<unsigned*>(workspace) + kNormBarrierWord;
    }
    // outputs by TMA tensor stores: box of 32 features x 128 tokens, 64-byte
    // swizzle (the kernel's staging layout)
    CUtensorMap tmY;
    std::memset(&tmY, 0, sizeof(tmY));
    a.use_tma_store = 0;
    if (a.vec_ok) {
      const uint64_t cols = silu ? (uint64_t)(N / 2) : (uint64_t)N;
      if (make_tmap_sw(&tmY, y, cols, (uint64_t)T, (uint64_t)ldy, 32, (uint32_t)kGemmBM,
                       CU_TENSOR_MAP_SWIZZLE_64B) == B200_OK)
        a.use_tma_store = 1;
    }
    return launch_pair(p, tmW, tmX, tmY, a, st, "gemm_pair_tcgen05_kernel");
  }
  const GemmPlan p = plan_gemm(ds, T, N, K, silu);
  CUtensorMap tmW, tmX;
  if (int r = make_tmap(&tmW, w, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, kGemmBK,
                        silu ? 64u : (uint32_t)kGemmBM))
    return r;
  if (int r = make_tmap(&tmX, x, (uint64_t)K, (uint64_t)T, (uint64_t)ldx, kGemmBK, (uint32_t)p.BN))
    return r;
  if (int r = ensure_smem(ds, 1u, gemm_tn_tcgen05_kernel, p.smem)) return r;
  GemmArgs a{};
  a.T = T; a.N = N; a.K = K; a.BN = p.BN; a.stages = p.stages; a.num_kb = p.num_kb;
  a.kb_per_split = p.kb_per_split; a.splits = p.splits; a.tmem_cols = p.tmem_cols;
  a.epi = silu ? EPI_SILU : EPI_BF16;
  a.vec_ok = aligned16(y) && (ldy % 8 == 0);
  a.y = static_cast<__nv_bfloat16*>(y); a.ldy = ldy;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.silu_inter = N / 2;
  a.err = ds->err;
  cudaLaunchConfig_t cfg = {};
  // token tiles fastest: the CTAs that share a W slab run side by side and the
  // second read of each W block hits L2
  cfg.gridDim = dim3(p.token_tiles, p.n_tiles, p.splits);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int nattr = 0;
  if (p.splits > 1) {
    attr[nattr].id = cudaLaunchAttributeClusterDimension;
    attr[nattr].val.clusterDim.x = 1;
    attr[nattr].val.clusterDim.y = 1;
    attr[nattr].val.clusterDim.z = p.splits;
    ++nattr;
  }
  if (pdl_enabled(true)) {
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr].val.programmaticStreamSerializationAllowed = 1;
    ++nattr;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_tn_tcgen05_kernel, tmW, tmX, a);
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "gemm launch: %s", cudaGetErrorString(e));
  return check_launch("gemm_tn_tcgen05_kernel");
}

// Plan of the fused RowParallelLinear launch: the single-SM GEMM plan with
// the largest K split (down to none) whose grid is co-resident, since owners
// wait for their peers' CTAs.  B200_ERR_UNSUPPORTED when no grid fits or the
// CTA positions exceed the flags.  Depends only on (T, N, K), the device type
// and `max_positions`, so every rank of a job gets the same answer.
int plan_allreduce(DeviceState* ds, int T, int N, int K, long long max_positions, GemmPlan* out) {
  GemmPlan p = plan_gemm(ds, T, N, K, false);
  if (int r = ensure_smem(ds, 1u, gemm_tn_tcgen05_kernel, p.smem)) return r;
  // co-resident CTAs for a split (occupancy queries are slow: cached per
  // device, split and shared-memory size)
  static long long resident_cache[kMaxDevices][9][4] = {};
  static int resident_smem[kMaxDevices][9][4] = {};
  int dev_id = 0;
  cudaGetDevice(&dev_id);
  auto resident_for = [&](int splits) -> long long {
    std::lock_guard<std::mutex> lock(g_host_mutex);
    for (int i = 0; i < 4; ++i)
      if (resident_smem[dev_id][splits][i] == p.smem) return resident_cache[dev_id][splits][i];
    const long long v = [&]() -> long long {
    if (splits == 1) {
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemm_tn_tcgen05_kernel, kGemmThreads,
                                                        p.smem) != cudaSuccess) {
        cudaGetLastError();
        per_sm = 0;
      }
      return (long long)per_sm * ds->num_sms;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, splits);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = p.smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = splits;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_tn_tcgen05_kernel, &cfg) != cudaSuccess) {
      cudaGetLastError();
      clusters = 0;
    }
    return (long long)clusters * splits;
    }();
    for (int i = 0; i < 4; ++i)
      if (resident_smem[dev_id][splits][i] == 0) {
        resident_smem[dev_id][splits][i] = p.smem;
        resident_cache[dev_id][splits][i] = v;
        break;
      }
    return v;
  };
  const long long tiles = (long long)p.n_tiles * p.token_tiles;
  int splits = p.splits;
  while (splits > 1 && tiles * splits > resident_for(splits)) --splits;
  if (splits != p.splits) {
    p.kb_per_split = (p.num_kb + splits - 1) / splits;
    p.splits = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;
  }
  const long long ctas = tiles * p.splits;
  if (ctas > max_positions)
    return fail(B200_ERR_UNSUPPORTED, "linear_allreduce: %lld CTA positions exceed the %lld flags", ctas, max_positions);
  const long long resident = resident_for(p.splits);
  if (ctas > resident)
    return fail(B200_ERR_UNSUPPORTED, "linear_allreduce: %lld CTAs cannot all be resident (%lld)", ctas, resident);
  *out = p;
  return B200_OK;
}

// Fused RowParallelLinear: GEMM + all-reduce in one launch (EPI_ALLREDUCE).
int run_gemm_allreduce(const void* x, long long ldx, const void* w, long long ldw, const void* bias,
                       int T, int N, int K, const AllReducePeers& ar, long long max_positions,
                       cudaStream_t st) {
  if (T <= 0) return B200_OK;
  if (N <= 0 || K <= 0 || N % 8) return fail(B200_ERR_INVALID, "linear_allreduce: N=%d must be a multiple of 8", N);
  if (K % 8 || ldx % 8 || ldw % 8 || ldx < K || ldw < K)
    return fail(B200_ERR_INVALID, "linear_allreduce: K and row strides must be multiples of 8");
  if (!aligned16(x) || !aligned16(w)) return fail(B200_ERR_INVALID, "linear_allreduce: x and w must be 16-byte aligned");
  if (ar.world < 1 || ar.world > kMaxTpRanks || ar.rank < 0 || ar.rank >= ar.world)
    return fail(B200_ERR_INVALID, "linear_allreduce: rank %d / world %d", ar.rank, ar.world);
  if (T > ar.stage_rows || ar.ldo < N || ar.ldo % 8)
    return fail(B200_ERR_UNSUPPORTED, "linear_allreduce: %d rows exceed the %lld staged rows (or ldo)", T, ar.stage_rows);
  for (int r = 0; r < ar.world; ++r)
    if (!ar.stage[r] || !ar.out[r] || !ar.flags[r] || !ar.done[r] || !aligned16(ar.stage[r]) ||
        !aligned16(ar.out[r]))
      return fail(B200_ERR_PEER, "linear_allreduce: peer buffers of rank %d are missing", r);
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  GemmPlan p{};
  if (int r = plan_allreduce(ds, T, N, K, max_positions, &p)) return r;
  CUtensorMap tmW, tmX;
  if (int r = make_tmap(&tmW, w, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, kGemmBK, (uint32_t)kGemmBM)) return r;
  if (int r = make_tmap(&tmX, x, (uint64_t)K, (uint64_t)T, (uint64_t)ldx, kGemmBK, (uint32_t)p.BN)) return r;
  GemmArgs a{};
  a.T = T; a.N = N; a.K = K; a.BN = p.BN; a.stages = p.stages; a.num_kb = p.num_kb;
  a.kb_per_split = p.kb_per_split; a.splits = p.splits; a.tmem_cols = p.tmem_cols;
  a.epi = EPI_ALLREDUCE;
  a.vec_ok = 1;
  a.y = nullptr; a.ldy = ar.ldo;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.err = ds->err;
  a.ar = ar;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.token_tiles, p.n_tiles, p.splits);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int nattr = 0;
  if (p.splits > 1) {
    attr[nattr].id = cudaLaunchAttributeClusterDimension;
    attr[nattr].val.clusterDim.x = 1;
    attr[nattr].val.clusterDim.y = 1;
    attr[nattr].val.clusterDim.z = p.splits;
    ++nattr;
  }
  if (pdl_enabled(true)) {
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr].val.programmaticStreamSerializationAllowed = 1;
    ++nattr;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_tn_tcgen05_kernel, tmW, tmX, a);
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "gemm allreduce launch: %s", cudaGetErrorString(e));
  return check_launch("gemm_tn_tcgen05_kernel(allreduce)");
}

}  // namespace

// ===========================================================================
// exported C-ABI
// ===========================================================================
extern "C" {

const char* b200_last_error(void) { return g_last_error.c_str(); }

int b200_version(void) { return B200_ABI_VERSION; }

unsigned long long b200_launch_count(void) { return g_launches; }

int b200_device_error(unsigned* out, int clear) {
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  unsigned v = 0;
  cudaError_t e = cudaMemcpy(&v, ds->err, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "read error word: %s", cudaGetErrorString(e));
  if (clear) {
    const unsigned z = 0;
    e = cudaMemcpy(ds->err, &z, sizeof(z), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return fail(B200_ERR_CUDA, "clear error word: %s", cudaGetErrorString(e));
  }
  if (out) *out = v;
  return B200_OK;
}

int b200_linear_workspace_bytes(int T, int N, int K, size_t* bytes) {
  if (!bytes || T < 0 || N <= 0 || K <= 0) return fail(B200_ERR_INVALID, "bad arguments");
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  // the persistent SM-pair kernel's split-K flags and partial tiles (the
  // same bound for every shape, so one buffer serves every GEMM)
  *bytes = pair_workspace_bytes(ds->num_sms);
  return B200_OK;
}

int b200_gemm_schedule_check(long long tiles, int num_kb, int max_pairs, int grouped) {
  if (tiles <= 0 || tiles > (1LL << 22) || num_kb <= 0 || num_kb > 4096 || max_pairs <= 0 ||
      max_pairs > 512 || tiles * num_kb > (1LL << 24))
    return fail(B200_ERR_INVALID, "schedule check: bad arguments");
  const PairSchedule sc = pair_schedule(tiles, num_kb, max_pairs, grouped != 0);
  std::string cover((size_t)(tiles * num_kb), '\0');
  long long bad = 0;
  if (sc.pairs < 1 || sc.pairs > max_pairs) ++bad;
  // flag area: 2 words per pair below the done counters, which fit the 4 KiB
  if (2 * sc.pairs > kGrpDoneOffset || kGrpDoneOffset + 2 * sc.split > 1024) ++bad;
  const long long total = tiles * num_kb;
  for (int pr = 0; pr < sc.pairs && pr >= 0; ++pr) {
    long long u = total * pr / sc.pairs;
    const long long u_end = total * (pr + 1) / sc.pairs;
    int k = 0;
    PairSeg sg;
    long long segs = 0;
    while (pair_next_seg(sc.sched, tiles, num_kb, sc.whole, sc.split, sc.group, pr, sc.pairs, u, u_end, k, sg)) {
      if (++segs > total + 1) return fail(B200_ERR_INVALID, "schedule check: pair %d does not terminate", pr);
      if (sg.tile < 0 || sg.tile >= tiles || sg.kbb < 0 || sg.kbe > num_kb || sg.kbb >= sg.kbe) {
        ++bad;
        continue;
      }
      // a grouped member is pair tile * g + member of a split tile
      if (sg.member >= 0 &&
          (sc.sched != 1 || sg.tile >= sc.split || sg.tile * sc.group + sg.member != pr || sg.member >= sc.group))
        ++bad;
      for (int kb = sg.kbb; kb < sg.kbe; ++kb) {
        char& c = cover[(size_t)(sg.tile * num_kb + kb)];
        if (c < 2) ++c;
      }
    }
  }
  for (char c : cover)
    if (c != 1) ++bad;
  return (int)std::min<long long>(bad, 1 << 30);
}

int b200_linear(const void* x, long long ldx, const void* w, long long ldw, const void* bias,
                void* y, long long ldy, int T, int N, int K, void* workspace, size_t ws_bytes,
                b200_stream_t stream) {
  return run_gemm(x, ldx, w, ldw, bias, y, ldy, T, N, K, false, workspace, ws_bytes,
                  reinterpret_cast<cudaStream_t>(stream));
}

int b200_linear_silu_and_mul(const void* x, long long ldx, const void* w, long long ldw, void* y,
                             long long ldy, int T, int I, int K, void* workspace, size_t ws_bytes,
                             b200_stream_t stream) {
  return run_gemm(x, ldx, w, ldw, nullptr, y, ldy, T, 2 * I, K, true, workspace, ws_bytes,
                  reinterpret_cast<cudaStream_t>(stream));
}

int b200_rmsnorm_linear(const void* x, long long ldx, const void* residual, void* residual_out,
                        const void* norm_weight, float eps, void* xn, long long ldxn, const void* w,
                        long long ldw, void* y, long long ldy, int T, int N, int K, int silu,
                        void* workspace, size_t ws_bytes, b200_stream_t stream) {
  if (T <= 0) return B200_OK;
  if (!x || !xn || !norm_weight || !w || !y)
    return fail(B200_ERR_INVALID, "rmsnorm_linear: null pointer");
  if (K <= 0 || K % 8 || K > 8192 || ldx % 8 || ldxn % 8 || ldx < K || ldxn < K || !aligned16(x) ||
      !aligned16(xn) || !aligned16(norm_weight))
    return fail(B200_ERR_INVALID, "rmsnorm_linear: K=%d (<= 8192, multiple of 8) and 16-byte aligned rows", K);
  if (residual && (!residual_out || !aligned16(residual) || !aligned16(residual_out)))
    return fail(B200_ERR_INVALID, "rmsnorm_linear: residual needs an aligned residual_out");
  NormIn nrm{x, ldx, residual, residual ? residual_out : nullptr, norm_weight, eps};
  return run_gemm(xn, ldxn, w, ldw, nullptr, y, ldy, T, N, K, silu != 0, workspace, ws_bytes,
                  reinterpret_cast<cudaStream_t>(stream), &nrm);
}

int b200_rms_norm(const void* x, long long x_stride, const void* residual, const void* weight,
                  void* out, long long out_stride, void* residual_out, int rows, int dim, float eps,
                  b200_stream_t stream) {
  return launch_rms_norm(x, x_stride, residual, weight, out, out_stride, residual_out, rows, dim, eps,
                         reinterpret_cast<cudaStream_t>(stream));
}

int b200_qk_norm_rope_store(const void* q_in, long long q_in_stride, const void* k_in,
                            long long k_in_stride, const void* v_in, long long v_in_stride, int T,
                            int Hq, int Hkv, const void* q_norm_w, const void* k_norm_w, float eps,
                            const float* cos_sin, long long max_pos, const long long* positions,
                            const int* slot_mapping, void* k_cache, void* v_cache,
                            long long num_slots, void* q_out, void* k_out, void* v_out,
                            b200_stream_t stream) {
  if (T <= 0) return B200_OK;
  if (Hq <= 0 || Hkv <= 0 || !q_in || !k_in || !q_out || !cos_sin || !positions)
    return fail(B200_ERR_INVALID, "qk_norm_rope_store: missing argument");
  if ((q_in_stride | k_in_stride | v_in_stride) % 2)
    return fail(B200_ERR_INVALID, "qk_norm_rope_store: strides must be even");
  if (k_cache && (!v_cache || !slot_mapping || !v_in))
    return fail(B200_ERR_INVALID, "qk_norm_rope_store: cache store needs v, v_cache and slot_mapping");
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  QKNormRopeArgs a{};
  a.q_in = static_cast<const __nv_bfloat16*>(q_in);
  a.k_in = static_cast<const __nv_bfloat16*>(k_in);
  a.v_in = static_cast<const __nv_bfloat16*>(v_in);
  a.q_in_stride = q_in_stride; a.k_in_stride = k_in_stride; a.v_in_stride = v_in_stride;
  a.T = T; a.Hq = Hq; a.Hkv = Hkv;
  a.q_w = static_cast<const __nv_bfloat16*>(q_norm_w);
  a.k_w = static_cast<const __nv_bfloat16*>(k_norm_w);
  a.eps = eps; a.cos_sin = cos_sin; a.positions = positions; a.max_pos = max_pos;
  a.slot_mapping = slot_mapping;
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.num_slots = num_slots;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.k_out = static_cast<__nv_bfloat16*>(k_out);
  a.v_out = static_cast<__nv_bfloat16*>(v_out);
  a.err = ds->err;
  const long long warps = (long long)T * (Hq + (v_in ? 2 : 1) * Hkv);
  const int blocks = (int)std::min<long long>((warps + 7) / 8, (long long)ds->num_sms * 16);
  launch_ex(qk_norm_rope_store_kernel, dim3(blocks), dim3(256), 0,
            reinterpret_cast<cudaStream_t>(stream), nullptr, 0, a);
  return check_launch("qk_norm_rope_store_kernel");
}

int b200_store_kvcache(const void* key, long long key_stride, const void* value,
                       long long value_stride, void* k_cache, void* v_cache,
                       const int* slot_mapping, int T, int D, long long num_slots,
                       b200_stream_t stream) {
  if (T <= 0) return B200_OK;
  if (D <= 0 || D % 8 || key_stride % 8 || value_stride % 8 || !aligned16(key) ||
      !aligned16(value) || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(B200_ERR_INVALID, "store_kvcache: D and strides must be multiples of 8 elements, 16-byte aligned");
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  const long long vecs = (long long)T * (D / 8);
  const int blocks = (int)std::min<long long>((vecs + 255) / 256, (long long)ds->num_sms * 8);
  launch_ex(store_kvcache_kernel, dim3(blocks), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
            nullptr, 0, static_cast<const __nv_bfloat16*>(key), key_stride,
            static_cast<const __nv_bfloat16*>(value), value_stride,
            static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache),
            slot_mapping, T, D, num_slots, ds->err);
  return check_launch("store_kvcache_kernel");
}

int b200_silu_and_mul(const void* x, long long x_stride, void* out, long long out_stride, int T,
                      int I, b200_stream_t stream) {
  if (T <= 0) return B200_OK;
  if (I <= 0 || I % 8 || x_stride % 8 || out_stride % 8 || !aligned16(x) || !aligned16(out))
    return fail(B200_ERR_INVALID, "silu_and_mul: I and strides must be multiples of 8");
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  const long long vecs = (long long)T * (I / 8);
  const int blocks = (int)std::min<long long>((vecs + 255) / 256, (long long)ds->num_sms * 8);
  launch_ex(silu_and_mul_kernel, dim3(blocks), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
            nullptr, 0, static_cast<const __nv_bfloat16*>(x), x_stride,
            static_cast<__nv_bfloat16*>(out), out_stride, T, I);
  return check_launch("silu_and_mul_kernel");
}

int b200_embedding(const long long* ids, const void* weight, void* out, int T, int H,
                   long long vocab_start, long long vocab_end, b200_stream_t stream) {
  if (T <= 0) return B200_OK;
  if (H <= 0 || H % 8 || !aligned16(weight) || !aligned16(out))
    return fail(B200_ERR_INVALID, "embedding: H must be a multiple of 8");
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  const long long vecs = (long long)T * (H / 8);
  const int blocks = (int)std::min<long long>((vecs + 255) / 256, (long long)ds->num_sms * 8);
  launch_ex(embedding_kernel, dim3(blocks), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
            nullptr, 0, ids, static_cast<const __nv_bfloat16*>(weight),
            static_cast<__nv_bfloat16*>(out), T, H, vocab_start, vocab_end, ds->err);
  return check_launch("embedding_kernel");
}

int b200_argmax(const void* logits, long long stride, int rows, int V, long long* out,
                b200_stream_t stream) {
  if (rows <= 0) return B200_OK;
  if (V <= 0) return fail(B200_ERR_INVALID, "argmax: V must be positive");
  launch_ex(argmax_kernel, dim3(rows), dim3(1024), 0, reinterpret_cast<cudaStream_t>(stream),
            nullptr, 0, static_cast<const __nv_bfloat16*>(logits), stride, V, out);
  return check_launch("argmax_kernel");
}

int b200_select_tokens_partial(const void* logits, long long stride, int rows, int V,
                               long long vocab_start, const float* temperatures, const float* noise,
                               long long noise_stride, unsigned long long seed,
                               unsigned long long offset, long long* keys, b200_stream_t stream) {
  if (rows <= 0) return B200_OK;
  if (V <= 0 || !logits || !keys || vocab_start < 0 || vocab_start + V > 0xFFFFFFFFll || stride < V ||
      (noise && noise_stride < V))
    return fail(B200_ERR_INVALID, "select_tokens_partial: rows=%d V=%d vocab_start=%lld", rows, V, vocab_start);
  SelectArgs a{};
  a.logits = static_cast<const __nv_bfloat16*>(logits);
  a.stride = stride;
  a.rows = rows;
  a.V = V;
  a.vocab_start = vocab_start;
  a.temperatures = temperatures;
  a.noise = noise;
  a.noise_stride = noise_stride;
  a.seed = seed;
  a.offset = offset;
  a.keys = keys;
  launch_ex(token_select_kernel, dim3(rows), dim3(1024), 0, reinterpret_cast<cudaStream_t>(stream), nullptr, 0,
            a);
  return check_launch("token_select_kernel");
}

namespace {
int exchange_args(int rank, int world, void* const* key_slots, void* const* flags, void* state,
                  long long max_rows, ExchangeArgs* x) {
  if (world < 1 || world > kXchgMaxRanks || rank < 0 || rank >= world || (world > 1 && (!flags || !state)))
    return fail(B200_ERR_INVALID, "exchange: rank %d / world %d / buffers", rank, world);
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  *x = ExchangeArgs{};
  x->rank = rank;
  x->world = world;
  x->max_rows = max_rows;
  x->state = static_cast<unsigned*>(state);
  x->err = ds->err;
  for (int r = 0; r < world && world > 1; ++r) {
    if (!flags[r]) return fail(B200_ERR_PEER, "exchange: flags of rank %d missing", r);
    x->flags[r] = static_cast<unsigned*>(flags[r]);
    if (key_slots) {
      if (!key_slots[r]) return fail(B200_ERR_PEER, "exchange: key slots of rank %d missing", r);
      x->key_slots[r] = static_cast<long long*>(key_slots[r]);
    }
  }
  return B200_OK;
}
}  // namespace

int b200_select_tokens_exchange(const long long* keys, int rows, int rank, int world,
                                void* const* key_slots, void* const* flags, void* state,
                                long long max_rows, long long* tokens, b200_stream_t stream) {
  if (rows <= 0) return B200_OK;
  if (!keys || !tokens || (world > 1 && (!key_slots || rows > max_rows)))
    return fail(B200_ERR_INVALID, "select_tokens_exchange: %d rows (at most max_rows %lld across ranks)", rows,
                max_rows);
  ExchangeArgs x;
  if (int r = exchange_args(rank, world, key_slots, flags, state, max_rows, &x)) return r;
  launch_ex(keys_exchange_kernel, dim3(1), dim3(1024), 0, reinterpret_cast<cudaStream_t>(stream), nullptr, 0,
            keys, rows, tokens, x);
  return check_launch("keys_exchange_kernel");
}

int b200_embedding_exchange(const long long* ids, const void* weight, int T, int H, long long vocab_start,
                            long long vocab_end, long long vocab_size, int rank, int world,
                            void* const* out, long long ld_out, void* const* flags, void* state,
                            b200_stream_t stream) {
  if (T <= 0) return B200_OK;
  if (!ids || !weight || !out || H <= 0 || H % 8 || ld_out % 8 || ld_out < H || !aligned16(weight))
    return fail(B200_ERR_INVALID, "embedding_exchange: H=%d ld_out=%lld", H, ld_out);
  ExchangeArgs x;
  if (int r = exchange_args(rank, world, nullptr, flags, state, 0, &x)) return r;
  __nv_bfloat16* const* outs = reinterpret_cast<__nv_bfloat16* const*>(out);
  for (int r = 0; r < world; ++r)
    if (!outs[r] || !aligned16(outs[r])) return fail(B200_ERR_PEER, "embedding_exchange: output of rank %d", r);
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  const long long vecs = (long long)T * (H / 8);
  const int blocks = (int)std::min<long long>((vecs + 255) / 256, (long long)ds->num_sms * 4);
  EmbeddingOuts o{};
  for (int r = 0; r < world; ++r) o.p[r] = outs[r];
  launch_ex(embedding_exchange_kernel, dim3(blocks), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), nullptr,
            0, ids, static_cast<const __nv_bfloat16*>(weight), T, H, vocab_start, vocab_end, vocab_size, o, ld_out,
            x);
  return check_launch("embedding_exchange_kernel");
}

int b200_step_metadata(const int* seq_info, const int* block_tables, int bt_stride, int B, int page,
                       long long* positions, int* slot_mapping, int* cu_seqlens_q, int* cu_seqlens_k,
                       int* context_lens, b200_stream_t stream) {
  if (B <= 0) return B200_OK;
  if (!seq_info || !positions || !cu_seqlens_q || !cu_seqlens_k || !context_lens || page <= 0 ||
      bt_stride < 0 || (bt_stride > 0 && (!block_tables || !slot_mapping)))
    return fail(B200_ERR_INVALID, "step_metadata: B=%d page=%d bt_stride=%d", B, page, bt_stride);
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  MetaArgs a{};
  a.start = seq_info;
  a.lq = seq_info + B;
  a.nblk = seq_info + 2 * B;
  a.block_tables = block_tables;
  a.bt_stride = bt_stride;
  a.B = B;
  a.page = page;
  a.positions = positions;
  a.slot_mapping = slot_mapping;
  a.cu_q = cu_seqlens_q;
  a.cu_k = cu_seqlens_k;
  a.context_lens = context_lens;
  a.err = ds->err;
  launch_ex(step_metadata_kernel, dim3(B), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), nullptr, 0, a);
  return check_launch("step_metadata_kernel");
}

int b200_attention_workspace_bytes(int max_seqs, int max_seqlen_k, int Hq, size_t* bytes) {
  if (!bytes || max_seqs < 0 || max_seqlen_k < 0 || Hq <= 0)
    return fail(B200_ERR_INVALID, "bad arguments");
  const size_t items = (size_t)max_seqs * ((max_seqlen_k + kDecItem - 1) / kDecItem);
  *bytes = (size_t)kDecSchedBytes + items * Hq * (kDecHD + 2) * sizeof(float);
  return B200_OK;
}

int b200_paged_attention(const void* q, long long q_stride, int num_q_rows, const void* k,
                         long long k_stride,
                         const void* v, long long v_stride, const void* k_cache,
                         const void* v_cache, long long num_slots, const int* block_tables,
                         int bt_stride, int bt_width, const int* cu_seqlens_q, const int* cu_seqlens_k, int B,
                         int max_seqlen_q, int max_seqlen_k, int Hq, int Hkv, int page,
                         float softmax_scale, void* out, long long out_stride, void* workspace,
                         size_t ws_bytes, b200_stream_t stream) {
  if (B <= 0 || max_seqlen_q <= 0) return B200_OK;
  if (Hq <= 0 || Hkv <= 0 || Hq % Hkv) return fail(B200_ERR_INVALID, "attention: Hq %% Hkv != 0");
  if (q_stride % 8 || out_stride % 8 || !aligned16(q) || !aligned16(out))
    return fail(B200_ERR_INVALID, "attention: q/out rows must be 16-byte aligned");
  if (block_tables && (!k_cache || !v_cache || page <= 0 || !aligned16(k_cache) || !aligned16(v_cache)))
    return fail(B200_ERR_INVALID, "attention: block tables need an aligned cache and page > 0");
  if (!block_tables && (!k || !v || k_stride % 8 || v_stride % 8 || !aligned16(k) || !aligned16(v)))
    return fail(B200_ERR_INVALID, "attention: contiguous K/V must be 16-byte aligned rows");
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int G = Hq / Hkv;
  const float scale_log2 = softmax_scale * 1.4426950408889634f;
  if (max_seqlen_q == 1 && block_tables && G <= 8 && B <= kDecMaxSeqs && Hkv <= kDecMaxKvHeads &&
      page % 256 == 0) {
    if (!workspace || ws_bytes <= (size_t)kDecSchedBytes || !aligned16(workspace))
      return fail(B200_ERR_WORKSPACE, "attention: decode workspace missing or too small");
    if (num_q_rows <= 0) return fail(B200_ERR_INVALID, "attention: num_q_rows must be positive");
    const size_t per_item = (size_t)Hq * (kDecHD + 2) * sizeof(float);
    CUtensorMap tmK, tmV, tmQ;
    const int qbox = Hq < 8 ? Hq : 8;
    if (int r = make_tmap_3d(&tmK, k_cache, kDecHD, Hkv, (uint64_t)num_slots, kDecHD * 2,
                             (uint64_t)Hkv * kDecHD * 2, 64, 1, kDecTile))
      return r;
    if (int r = make_tmap_3d(&tmV, v_cache, kDecHD, Hkv, (uint64_t)num_slots, kDecHD * 2,
                             (uint64_t)Hkv * kDecHD * 2, 64, 1, kDecTile))
      return r;
    if (int r = make_tmap_3d(&tmQ, q, kDecHD, Hq, (uint64_t)num_q_rows, kDecHD * 2,
                             (uint64_t)q_stride * 2, 64, (uint32_t)qbox, 1))
      return r;
    DecodeArgs a{};
    a.block_tables = block_tables; a.bt_stride = bt_stride; a.bt_width = bt_width;
    a.cu_q = cu_seqlens_q; a.cu_k = cu_seqlens_k;
    a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.G = G; a.page = page; a.q_box_rows = qbox;
    a.num_slots = num_slots;
    a.scale_log2 = scale_log2;
    a.sched = static_cast<int*>(workspace);
    a.cap_items = (long long)((ws_bytes - kDecSchedBytes) / per_item);
    a.part_ml = reinterpret_cast<float*>(static_cast<char*>(workspace) + kDecSchedBytes);
    a.part_o = a.part_ml + (size_t)a.cap_items * Hq * 2;
    a.out = static_cast<__nv_bfloat16*>(out); a.out_stride = out_stride;
    a.err = ds->err;
    const int smem = dec_smem_bytes();
    if (int r = ensure_smem(ds, 2u, decode_attn_kernel, smem)) return r;
    if (int r = launch_decode(ds, tmK, tmV, tmQ, a, smem, st)) return r;
    return check_launch("decode_attn_kernel");
  }
  // prefill on the tensor cores (tcgen05): 128-key tiles must not straddle
  // pages; B200_PREFILL=legacy selects the mma.sync kernel below
  const char* pf = getenv("B200_PREFILL");
  const bool legacy = pf && std::strcmp(pf, "legacy") == 0;
  if (!legacy && (!block_tables || page % kPtBN == 0) && num_q_rows > 0) {
    CUtensorMap tmQ, tmK, tmV;
    int r = make_tmap_3d(&tmQ, q, 128, Hq, (uint64_t)num_q_rows, 256, (uint64_t)q_stride * 2, 64, 1, kPtBM);
    if (!r) {
      if (block_tables) {
        r = make_tmap_3d(&tmK, k_cache, 128, Hkv, (uint64_t)num_slots, 256, (uint64_t)Hkv * 256, 64, 1, kPtBN);
        if (!r)
          r = make_tmap_3d(&tmV, v_cache, 128, Hkv, (uint64_t)num_slots, 256, (uint64_t)Hkv * 256, 64, 1, kPtBN);
      } else {
        // without a block table K / V are per token, num_q_rows rows (the
        // reference's fresh prefill: cu_seqlens_k == cu_seqlens_q)
        r = make_tmap_3d(&tmK, k, 128, Hkv, (uint64_t)num_q_rows, 256, (uint64_t)k_stride * 2, 64, 1, kPtBN);
        if (!r) r = make_tmap_3d(&tmV, v, 128, Hkv, (uint64_t)num_q_rows, 256, (uint64_t)v_stride * 2, 64, 1, kPtBN);
      }
    }
    if (r) return r;
    PrefillTcArgs t{};
    t.cu_q = cu_seqlens_q; t.cu_k = cu_seqlens_k;
    t.block_tables = block_tables; t.bt_stride = bt_stride; t.bt_width = bt_width;
    t.num_slots = num_slots;
    t.B = B; t.Hq = Hq; t.Hkv = Hkv; t.G = G; t.page = page > 0 ? page : 1;
    t.scale_log2 = scale_log2;
    t.out = static_cast<__nv_bfloat16*>(out); t.out_stride = out_stride;
    t.err = ds->err;
    if (int rr = ensure_smem(ds, 16u, prefill_tc_kernel, kPtSmemBytes)) return rr;
    dim3 grid((max_seqlen_q + kPtBM - 1) / kPtBM, Hq, B);
    const cudaError_t e = launch_ex(prefill_tc_kernel, grid, dim3(kPtThreads), kPtSmemBytes, st, nullptr, 0,
                                    tmQ, tmK, tmV, t);
    if (e != cudaSuccess) return fail(B200_ERR_CUDA, "prefill_tc launch: %s", cudaGetErrorString(e));
    return check_launch("prefill_tc_kernel");
  }
  PrefillArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q); a.q_stride = q_stride;
  a.k = static_cast<const __nv_bfloat16*>(k); a.v = static_cast<const __nv_bfloat16*>(v);
  a.k_stride = k_stride; a.v_stride = v_stride;
  a.k_cache = block_tables ? static_cast<const __nv_bfloat16*>(k_cache) : nullptr;
  a.v_cache = block_tables ? static_cast<const __nv_bfloat16*>(v_cache) : nullptr;
  a.block_tables = block_tables; a.bt_stride = bt_stride; a.bt_width = bt_width; a.num_slots = num_slots;
  a.cu_q = cu_seqlens_q; a.cu_k = cu_seqlens_k;
  a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.G = G; a.page = page;
  a.scale_log2 = scale_log2;
  a.out = static_cast<__nv_bfloat16*>(out); a.out_stride = out_stride;
  a.err = ds->err;
  const int smem = 16384 + 2 * 32768;
  if (int r = ensure_smem(ds, 4u, prefill_attn_kernel, smem)) return r;
  dim3 grid((max_seqlen_q + kPfBM - 1) / kPfBM, Hq, B);
  launch_ex(prefill_attn_kernel, grid, dim3(128), smem, st, nullptr, 0, a);
  return check_launch("prefill_attn_kernel");
}

int b200_ipc_export(const void* ptr, void* handle, unsigned long long* offset) {
  if (!ptr || !handle || !offset) return fail(B200_ERR_INVALID, "ipc_export: null argument");
  auto range = address_range_fn();
  if (!range) return fail(B200_ERR_CUDA, "cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(B200_ERR_CUDA, "ipc_export: pointer is not device memory");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle, &h, sizeof(h));
  *offset = (unsigned long long)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return B200_OK;
}

int b200_ipc_import(const void* handle, unsigned long long offset, void** ptr) {
  if (!handle || !ptr) return fail(B200_ERR_INVALID, "ipc_import: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *ptr = static_cast<char*>(base) + offset;
  return B200_OK;
}

int b200_ipc_close(void* ptr, unsigned long long offset) {
  if (!ptr) return B200_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return B200_OK;
}

int b200_linear_allreduce_supported(int T, int N, int K, int world, long long stage_rows,
                                    long long ldo, long long max_positions, int* supported) {
  if (!supported) return fail(B200_ERR_INVALID, "linear_allreduce_supported: null result");
  *supported = 0;
  if (T <= 0 || N <= 0 || K <= 0 || N % 8 || K % 8 || world < 1 || world > kMaxTpRanks)
    return fail(B200_ERR_INVALID, "linear_allreduce_supported: T=%d N=%d K=%d world=%d", T, N, K, world);
  if (T > stage_rows || ldo < N || ldo % 8) {
    fail(B200_ERR_UNSUPPORTED, "linear_allreduce: %d rows exceed the %lld staged rows (or ldo)", T, stage_rows);
    return B200_OK;
  }
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  GemmPlan p{};
  const int r = plan_allreduce(ds, T, N, K, max_positions, &p);
  if (r == B200_ERR_UNSUPPORTED) return B200_OK;  // *supported stays 0; the reason is the last error
  if (r) return r;
  *supported = 1;
  return B200_OK;
}

int b200_linear_allreduce(const void* x, long long ldx, const void* w, long long ldw,
                          const void* bias, int T, int N, int K, int rank, int world,
                          void* const* stage, void* const* out, void* const* flags,
                          void* const* done, long long stage_rows, long long ldo,
                          long long max_positions, int one_shot, b200_stream_t stream) {
  if (world < 1 || world > kMaxTpRanks || !stage || !out || !flags || !done)
    return fail(B200_ERR_INVALID, "linear_allreduce: world %d / peer arrays", world);
  AllReducePeers ar{};
  ar.rank = rank;
  ar.world = world;
  ar.stage_rows = stage_rows;
  ar.ldo = ldo;
  ar.oneshot = one_shot ? 1 : 0;
  ar.positions = max_positions;
  for (int r = 0; r < world; ++r) {
    ar.stage[r] = static_cast<__nv_bfloat16*>(stage[r]);
    ar.out[r] = static_cast<__nv_bfloat16*>(out[r]);
    ar.flags[r] = static_cast<unsigned*>(flags[r]);
    ar.done[r] = static_cast<unsigned*>(done[r]);
  }
  return run_gemm_allreduce(x, ldx, w, ldw, bias, T, N, K, ar, max_positions,
                            reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ===========================================================================
// Allocation-free decode attention
//
// Some callers cannot hand this library a workspace: a host runtime that
// reaches these kernels through a foreign-function boundary (cgo, JNI,
// ctypes) with device memory owned by another allocator, or a serving loop
// that must never call cudaMalloc -- cudaMalloc can synchronise the device
// and stall every stream, and it cannot be recorded into a CUDA graph.  For
// them b200_paged_decode_attention_static keeps the decode kernel's scratch
// (the scheduler counters and the split-KV partials) in the fixed array below.  The array is part of the library
// image: every GPU that loads libb200ops.so holds these 32 MiB until the
// process exits.
// ===========================================================================
namespace {

constexpr size_t kStaticDecodeScratchBytes = size_t(32) << 20;
static __device__ __align__(256) unsigned char g_static_decode_scratch[kStaticDecodeScratchBytes];

// Device address of the array on the current device, looked up once per
// device (host code may not use the symbol itself as a device pointer).
int static_decode_scratch(void** out) {
  static void* addr[kMaxDevices] = {};
  std::lock_guard<std::mutex> lock(g_host_mutex);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(B200_ERR_INVALID, "device %d out of range", dev);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_decode_scratch);
    if (e != cudaSuccess)
      return fail(B200_ERR_CUDA, "scratch symbol address: %s", cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return B200_OK;
}

}  // namespace

extern "C" int b200_paged_decode_attention_static(
    const void* q, long long q_stride, int num_q_rows, const void* k_cache, const void* v_cache,
    long long num_slots, const int* block_tables, int bt_stride, int bt_width,
    const int* cu_seqlens_q, const int* cu_seqlens_k, int B, int max_seqlen_k, int Hq, int Hkv,
    int page, float softmax_scale, void* out, long long out_stride, b200_stream_t stream) {
  if (B <= 0) return B200_OK;
  if (Hq <= 0 || Hkv <= 0 || Hq % Hkv || Hq / Hkv > 8 || Hkv > kDecMaxKvHeads || B > kDecMaxSeqs)
    return fail(B200_ERR_UNSUPPORTED,
                "decode_static: needs Hq %% Hkv == 0, Hq/Hkv <= 8, Hkv <= %d, B <= %d", kDecMaxKvHeads,
                kDecMaxSeqs);
  if (!q || !k_cache || !v_cache || !block_tables || !cu_seqlens_q || !cu_seqlens_k || !out ||
      page <= 0 || page % 256 || num_q_rows <= 0 || max_seqlen_k < 0)
    return fail(B200_ERR_INVALID, "decode_static: missing argument or page not a multiple of 256");
  if (q_stride % 8 || out_stride % 8 || !aligned16(q) || !aligned16(out) || !aligned16(k_cache) ||
      !aligned16(v_cache))
    return fail(B200_ERR_INVALID, "decode_static: rows must be 16-byte aligned");
  const size_t per_item = (size_t)Hq * (kDecHD + 2) * sizeof(float);
  const size_t items = (size_t)B * ((max_seqlen_k + kDecItem - 1) / kDecItem);
  const size_t need = (size_t)kDecSchedBytes + items * per_item;
  if (need > kStaticDecodeScratchBytes)
    return fail(B200_ERR_WORKSPACE,
                "decode_static: %d sequences of up to %d keys with %d heads need %zu bytes of scratch; "
                "the fixed array holds %zu",
                B, max_seqlen_k, Hq, need, kStaticDecodeScratchBytes);
  DeviceState* ds;
  if (int r = device_state(&ds)) return r;
  void* scratch = nullptr;
  if (int r = static_decode_scratch(&scratch)) return r;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // the scheduler counters must start at zero; a call that ended early must
  // not leave stale counts for this one
  cudaError_t e = cudaMemsetAsync(scratch, 0, kDecSchedBytes, st);
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "decode_static: clear: %s", cudaGetErrorString(e));
  CUtensorMap tmK, tmV, tmQ;
  const int qbox = Hq < 8 ? Hq : 8;
  if (int r = make_tmap_3d(&tmK, k_cache, kDecHD, Hkv, (uint64_t)num_slots, kDecHD * 2,
                           (uint64_t)Hkv * kDecHD * 2, 64, 1, kDecTile))
    return r;
  if (int r = make_tmap_3d(&tmV, v_cache, kDecHD, Hkv, (uint64_t)num_slots, kDecHD * 2,
                           (uint64_t)Hkv * kDecHD * 2, 64, 1, kDecTile))
    return r;
  if (int r = make_tmap_3d(&tmQ, q, kDecHD, Hq, (uint64_t)num_q_rows, kDecHD * 2,
                           (uint64_t)q_stride * 2, 64, (uint32_t)qbox, 1))
    return r;
  DecodeArgs a{};
  a.block_tables = block_tables; a.bt_stride = bt_stride; a.bt_width = bt_width;
  a.cu_q = cu_seqlens_q; a.cu_k = cu_seqlens_k;
  a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.G = Hq / Hkv; a.page = page; a.q_box_rows = qbox;
  a.num_slots = num_slots;
  a.scale_log2 = softmax_scale * 1.4426950408889634f;
  a.sched = static_cast<int*>(scratch);
  a.cap_items = (long long)((kStaticDecodeScratchBytes - kDecSchedBytes) / per_item);
  a.part_ml = reinterpret_cast<float*>(static_cast<char*>(scratch) + kDecSchedBytes);
  a.part_o = a.part_ml + (size_t)a.cap_items * Hq * 2;
  a.out = static_cast<__nv_bfloat16*>(out); a.out_stride = out_stride;
  a.err = ds->err;
  const int smem = dec_smem_bytes();
  if (int r = ensure_smem(ds, 2u, decode_attn_kernel, smem)) return r;
  if (int r = launch_decode(ds, tmK, tmV, tmQ, a, smem, st)) return r;
  return check_launch("decode_attn_kernel");
}
