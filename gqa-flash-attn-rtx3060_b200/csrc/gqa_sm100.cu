// libgqa_sm100.so: host side of the C ABI declared in include/gqa_sm100.h.
//
// Validates arguments (returning GQA_ERR_* before any launch), builds the TMA
// tensor maps, sizes the launch for the current device's SM count and
// enqueues the kernels on the caller's stream. Nothing here allocates device
// memory or synchronises (except gqa_device_error and the peer exchange's setup
// calls, gqa_exchange_alloc / gqa_ipc_*, which say so).
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "gqa_common.cuh"
#include "gqa_cache.cuh"
#include "gqa_combine.cuh"
#include "gqa_prefill.cuh"
#include "gqa_stream.cuh"

namespace gqa {
namespace {

// ----------------------------------------------------------------------------- device cache
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct DeviceState {
  bool ready = false;
  int status = GQA_OK;
  int sm_count = 0;
};

// The prefill kernel rebalances registers with setmaxnreg; the increase can only
// be granted if the launch reserved enough registers (threads x registers per
// thread). Refuse to launch a build where that does not hold: the request would
// never be granted and the kernel would not finish.
template <typename K>
int check_reg_split(K kernel, int threads, int needed) {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, kernel) != cudaSuccess) return GQA_ERR_CUDA;
  return (a.numRegs * threads >= needed) ? GQA_OK : GQA_ERR_UNSUPPORTED;
}

std::mutex g_mutex;
std::vector<DeviceState> g_devices;
EncodeTiledFn g_encode = nullptr;

template <typename K>
cudaError_t set_smem(K kernel, int bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

int init_device(int dev) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return GQA_ERR_CUDA;
  if (prop.major != 10) return GQA_ERR_NO_DEVICE;
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      return GQA_ERR_CUDA;
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  cudaError_t e = cudaSuccess;
  auto chk = [&](cudaError_t x) { if (x != cudaSuccess && e == cudaSuccess) e = x; };
  int rs = GQA_OK;
  // Both key-split instantiations of each (head_dim, dtype): shared memory opt-in,
  // and the setmaxnreg split must fit the registers the launch holds.
#define GQA_PREP_PREFILL(HD, BF, SP)                                                      \
  chk(set_smem(gqa_prefill_kernel<HD, BF, SP>, PrefillCfg<HD>::kSmemBytes));              \
  if (!rs) rs = check_reg_split(gqa_prefill_kernel<HD, BF, SP>, PrefillCfg<HD>::kThreads, \
                                PrefillCfg<HD>::kRegsNeeded)
#define GQA_PREP_PREFILL_PG(HD, BF, SP)                                                         \
  chk(set_smem(gqa_prefill_kernel<HD, BF, SP, true>, PrefillCfg<HD>::kSmemBytes));              \
  if (!rs) rs = check_reg_split(gqa_prefill_kernel<HD, BF, SP, true>, PrefillCfg<HD>::kThreads, \
                                PrefillCfg<HD>::kRegsNeeded)
  GQA_PREP_PREFILL(128, true, false); GQA_PREP_PREFILL(128, false, false);
  GQA_PREP_PREFILL(64, true, false); GQA_PREP_PREFILL(64, false, false);
  GQA_PREP_PREFILL(128, true, true); GQA_PREP_PREFILL(128, false, true);
  GQA_PREP_PREFILL(64, true, true); GQA_PREP_PREFILL(64, false, true);
  // Paged-cache instantiations (chunked prefill over vLLM-layout blocks).
  GQA_PREP_PREFILL_PG(128, true, false); GQA_PREP_PREFILL_PG(128, false, false);
  GQA_PREP_PREFILL_PG(64, true, false); GQA_PREP_PREFILL_PG(64, false, false);
  GQA_PREP_PREFILL_PG(128, true, true); GQA_PREP_PREFILL_PG(128, false, true);
  GQA_PREP_PREFILL_PG(64, true, true); GQA_PREP_PREFILL_PG(64, false, true);
#undef GQA_PREP_PREFILL
#undef GQA_PREP_PREFILL_PG
  if (e != cudaSuccess) return GQA_ERR_CUDA;
  if (rs) return rs;
#define GQA_SET_STREAM(HD, BF, RG) chk(set_smem(gqa_stream_kernel<HD, BF, RG>, StreamCfg<HD>::kSmemBytes))
  GQA_SET_STREAM(128, true, 1); GQA_SET_STREAM(128, true, 2); GQA_SET_STREAM(128, true, 4);
  GQA_SET_STREAM(128, false, 1); GQA_SET_STREAM(128, false, 2); GQA_SET_STREAM(128, false, 4);
  GQA_SET_STREAM(64, true, 1); GQA_SET_STREAM(64, true, 2); GQA_SET_STREAM(64, true, 4);
  GQA_SET_STREAM(64, false, 1); GQA_SET_STREAM(64, false, 2); GQA_SET_STREAM(64, false, 4);
#undef GQA_SET_STREAM
#define GQA_SET_STREAM_F8(BF, RG) chk(set_smem(gqa_stream_kernel<128, BF, RG, true>, StreamCfg<64>::kSmemBytes))
  GQA_SET_STREAM_F8(true, 1); GQA_SET_STREAM_F8(true, 2); GQA_SET_STREAM_F8(true, 4);
  GQA_SET_STREAM_F8(false, 1); GQA_SET_STREAM_F8(false, 2); GQA_SET_STREAM_F8(false, 4);
#undef GQA_SET_STREAM_F8
  // The transposed (keys x rows) decode instantiations.
  chk(set_smem(gqa_stream_kernel<128, true, 1, true, true>, StreamCfg<64>::kSmemBytes));
  chk(set_smem(gqa_stream_kernel<128, false, 1, true, true>, StreamCfg<64>::kSmemBytes));
  chk(set_smem(gqa_stream_kernel<128, true, 1, false, true>, StreamCfg<128>::kSmemBytes));
  chk(set_smem(gqa_stream_kernel<128, false, 1, false, true>, StreamCfg<128>::kSmemBytes));
  chk(set_smem(gqa_stream_kernel<64, true, 1, false, true>, StreamCfg<64>::kSmemBytes));
  chk(set_smem(gqa_stream_kernel<64, false, 1, false, true>, StreamCfg<64>::kSmemBytes));
  if (e != cudaSuccess) return GQA_ERR_CUDA;
  return GQA_OK;
}

// Returns GQA_OK and the SM count of the current device, initialising it once.
int current_device(int* sm_count) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GQA_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_mutex);
  if ((int)g_devices.size() <= dev) g_devices.resize(dev + 1);
  DeviceState& st = g_devices[dev];
  if (!st.ready) {
    st.status = init_device(dev);
    if (st.status == GQA_OK) {
      if (cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        st.status = GQA_ERR_CUDA;
    }
    st.ready = true;
  }
  if (sm_count) *sm_count = st.sm_count;
  return st.status;
}

// ----------------------------------------------------------------------------- validation
struct Shape {
  int batch, hq, hkv, group, seq_q, seq_kv, head_dim;
};

int check_shape(int batch, int hq, int hkv, int seq_q, int seq_kv, int head_dim, Shape* s) {
  if (batch < 0 || hq <= 0 || hkv <= 0 || seq_q < 0 || seq_kv < 0) return GQA_ERR_INVALID_ARG;
  if (hq % hkv != 0) return GQA_ERR_INVALID_ARG;
  if (head_dim != 64 && head_dim != 128) return GQA_ERR_UNSUPPORTED;
  const int g = hq / hkv;
  if (g > 128 || (g & (g - 1)) != 0) return GQA_ERR_UNSUPPORTED;  // packed tiles need a power-of-two group
  *s = Shape{batch, hq, hkv, g, seq_q, seq_kv, head_dim};
  return GQA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// (b, h, s, d) strides of a 16-bit tensor: d stride 1, the others multiples of 8 elements.
int check_strides(const void* ptr, const int64_t* st) {
  if (!ptr || !st) return GQA_ERR_INVALID_ARG;
  if (!aligned16(ptr)) return GQA_ERR_ALIGNMENT;
  if (st[3] != 1) return GQA_ERR_ALIGNMENT;
  for (int i = 0; i < 3; ++i)
    if (st[i] < 0 || (st[i] % 8) != 0) return GQA_ERR_ALIGNMENT;
  return GQA_OK;
}

// 4-D tensor map over a (b, h, s, d) 16-bit tensor (8-bit with `u8`), box {128 bytes of d,
// box_s, box_h, 1}, 128-byte swizzle. Strides are in elements.
int make_map(CUtensorMap* map, const void* ptr, const int64_t* st, int b, int h, int s, int d, int box_s,
             int box_h, bool u8 = false) {
  const cuuint64_t es = u8 ? 1 : 2;
  cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)s, (cuuint64_t)h, (cuuint64_t)b};
  cuuint64_t strides[3] = {(cuuint64_t)st[2] * es, (cuuint64_t)st[1] * es, (cuuint64_t)st[0] * es};
  // Degenerate strides (size-1 dims) may be 0 in caller metadata; TMA wants a valid stride.
  if (s == 1 && strides[0] == 0) strides[0] = (cuuint64_t)d * es;
  if (h == 1 && strides[1] == 0) strides[1] = strides[0] * s;
  if (b == 1 && strides[2] == 0) strides[2] = strides[1] * h;
  for (int i = 0; i < 3; ++i)
    if (strides[i] == 0 || (strides[i] & 15) != 0 || strides[i] >= (1ull << 40)) return GQA_ERR_ALIGNMENT;
  cuuint32_t box[4] = {u8 ? 128u : 64u, (cuuint32_t)box_s, (cuuint32_t)box_h, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = g_encode(map, u8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 4,
                        const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? GQA_OK : GQA_ERR_CUDA;
}

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

// Launch with programmatic stream serialisation: the kernel may begin while the
// previous kernel on the stream finishes; it calls pdl_wait() before any global
// memory access, so stream order holds for every byte it reads or writes.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, int threads, int smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ----------------------------------------------------------------------------- streaming plan
// Number of packed rows (group * block_m) the streaming kernel handles per unit.
constexpr int kStreamMaxRows = 64;
constexpr int kStreamCtasPerSm = 1;
constexpr int kMaxSplits = 64;

struct StreamPlan {
  int block_m, rows, rg, n_mtiles, units, nsplit, chunk;
};

StreamPlan plan_stream(const Shape& s, int sm_count, bool allow_split) {
  StreamPlan pl{};
  pl.block_m = std::max(1, std::min(s.seq_q, kStreamMaxRows / s.group));
  pl.rows = s.group * pl.block_m;
  pl.rg = pl.rows <= 16 ? 1 : (pl.rows <= 32 ? 2 : 4);
  pl.n_mtiles = (s.seq_q + pl.block_m - 1) / pl.block_m;
  pl.units = s.batch * s.hkv * pl.n_mtiles;
  const int stages = std::max(1, (s.seq_kv + 63) / 64);
  pl.nsplit = 1;
  pl.chunk = stages * 64;
  if (!allow_split) return pl;
  // Cost of a plan in units of one 64-key stage of streaming: every wave of CTAs
  // takes its chunk's stages plus a fixed per-CTA cost (set-up, pipeline ramp,
  // publishing the partial), about kFixedStages. Fewer waves beat a finer
  // balance: a second wave restarts the ramp.
  constexpr double kFixedStages = 5.0;
  const double slots = (double)sm_count * kStreamCtasPerSm;
  double best = 1e300;
  const int max_ns = std::min(std::min(stages, kMaxSplits), std::max(1, 4096 / pl.rows));
  for (int ns = 1; ns <= max_ns; ++ns) {
    const int chunk_st = (stages + ns - 1) / ns;
    const int ns_eff = (stages + chunk_st - 1) / chunk_st;
    if (ns_eff != ns) continue;
    const double waves = std::ceil((double)pl.units * ns_eff / slots);
    const double cost = waves * (chunk_st + kFixedStages);
    if (cost < best - 1e-9) {
      best = cost;
      pl.nsplit = ns;
      pl.chunk = chunk_st * 64;
    }
  }
  return pl;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t stream_ws_bytes(const StreamPlan& pl, int head_dim) {
  const size_t n = (size_t)pl.units * pl.nsplit * pl.rows;
  return align256(n * 4) * 2 + align256(n * head_dim * 4) + align256((size_t)pl.units * 4);
}

void stream_ws_carve(const StreamPlan& pl, int head_dim, void* ws, StreamParams* p) {
  const size_t n = (size_t)pl.units * pl.nsplit * pl.rows;
  uint8_t* c = reinterpret_cast<uint8_t*>(ws);
  p->ws_m = reinterpret_cast<float*>(c);
  c += align256(n * 4);
  p->ws_l = reinterpret_cast<float*>(c);
  c += align256(n * 4);
  p->ws_acc = reinterpret_cast<float*>(c);
  c += align256(n * head_dim * 4);
  p->ws_cnt = reinterpret_cast<unsigned*>(c);
}

bool use_stream(const Shape& s) { return s.group <= kStreamMaxRows && s.group * s.seq_q <= kStreamMaxRows; }

// ----------------------------------------------------------------------------- prefill plan
// Units are query pairs (2 x 128 packed rows) of one (batch, kv head). When they
// are fewer than the SMs (short query blocks against long keys, or a GPU's share
// of a sharded batch), each unit's key tiles are split across CTAs so every SM
// gets work; the partials are combined by the unit's last CTA.
struct PrefillPlan {
  int bm, n_pairs, units, nsplit, chunk_tiles, head_major;
};

// Key tiles a causal query pair starting at position p0 may see.
int pair_tiles(const Shape& s, int bm, int p0, bool causal) {
  int kv_end = s.seq_kv;
  if (causal) kv_end = std::min(kv_end, std::min(p0 + 2 * bm, s.seq_q) + s.seq_kv - s.seq_q);
  return std::max(0, (kv_end + 127) / 128);
}

PrefillPlan plan_prefill(const Shape& s, int sm_count, bool causal = true) {
  PrefillPlan pl{};
  pl.bm = 128 / s.group;
  const int n_tiles = (s.seq_q + pl.bm - 1) / pl.bm;
  pl.n_pairs = (n_tiles + 1) / 2;
  // Head-major order when every pair of a head has at least half the longest pair's
  // key tiles (chunked prefill against a longer cache, non-causal calls): measured on
  // B200, 2-8 % faster there (the heads' keys stay in L2 across their pairs), while
  // a full causal prefill needs the longest-first order for its tail (2K causal: 24 %
  // slower head-major).
  const int longest = pair_tiles(s, pl.bm, (pl.n_pairs - 1) * 2 * pl.bm, causal);
  const int shortest = pair_tiles(s, pl.bm, 0, causal);
  pl.head_major = (pl.n_pairs > 1 && 2 * shortest >= longest) ? 1 : 0;
  pl.units = pl.n_pairs * s.batch * s.hkv;
  pl.nsplit = 1;
  pl.chunk_tiles = 0;
  const int nk_max = (s.seq_kv + 127) / 128;
  if (pl.units > 0 && pl.units < sm_count) {
    int ns = std::min(sm_count / pl.units, 16);
    while (ns > 1 && nk_max < 2 * ns) --ns;  // at least two key tiles per split
    if (ns > 1) {
      pl.nsplit = ns;
      pl.chunk_tiles = (nk_max + ns - 1) / ns;
    }
  }
  return pl;
}

size_t prefill_ws_bytes(const PrefillPlan& pl, int head_dim) {
  if (pl.nsplit <= 1) return 0;
  const size_t rows = (size_t)pl.units * pl.nsplit * 256;
  return align256((size_t)pl.units * 4) + 2 * align256(rows * 4) + align256(rows * head_dim * 4);
}

void prefill_ws_carve(const PrefillPlan& pl, int head_dim, void* ws, PrefillParams* p) {
  const size_t rows = (size_t)pl.units * pl.nsplit * 256;
  uint8_t* c = reinterpret_cast<uint8_t*>(ws);
  p->ws_cnt = reinterpret_cast<unsigned*>(c);
  c += align256((size_t)pl.units * 4);
  p->ws_m = reinterpret_cast<float*>(c);
  c += align256(rows * 4);
  p->ws_l = reinterpret_cast<float*>(c);
  c += align256(rows * 4);
  p->ws_acc = reinterpret_cast<float*>(c);
  (void)head_dim;
}

template <int HD, bool BF, bool F8 = false>
cudaError_t launch_stream_hd(const StreamParams& p, const StreamPlan& pl, const CUtensorMap& km,
                             const CUtensorMap& vm, cudaStream_t st) {
  using Cfg = StreamCfg<F8 ? 64 : HD>;
  const dim3 grid(pl.units * pl.nsplit);
  const int smem = Cfg::kSmemBytes;
  if (pl.rows <= 8)  // decode: the transposed (keys x rows) MMA form
    return launch_pdl(gqa_stream_kernel<HD, BF, 1, F8, true>, grid, Cfg::kThreads, smem, st, p, km, vm);
  switch (pl.rg) {
    case 1: return launch_pdl(gqa_stream_kernel<HD, BF, 1, F8>, grid, Cfg::kThreads, smem, st, p, km, vm);
    case 2: return launch_pdl(gqa_stream_kernel<HD, BF, 2, F8>, grid, Cfg::kThreads, smem, st, p, km, vm);
    default: return launch_pdl(gqa_stream_kernel<HD, BF, 4, F8>, grid, Cfg::kThreads, smem, st, p, km, vm);
  }
}

// Fills the common fields of StreamParams and launches. With `paged`, k/v are paged
// caches (num_blocks, block_size, hkv, D) and their maps are (D, hkv, block_size,
// num_blocks) with {64, 1, 64, 1} boxes: the same 64-key x 128-byte smem tiles.
struct PagedCache {
  int block_size, num_blocks;
  bool fp8 = false;  // e4m3 K/V (head_dim 128)
};

int run_stream(const Shape& s, const StreamPlan& pl, StreamParams p, const void* k, const void* v,
               const int64_t* ks, const int64_t* vs, int dtype, cudaStream_t st, const PagedCache* paged = nullptr) {
  CUtensorMap km, vm;
  int rc;
  if (paged) {
    const int64_t cs[4] = {(int64_t)paged->block_size * s.hkv * s.head_dim, (int64_t)s.hkv * s.head_dim,
                           s.head_dim, 1};
    rc = make_map(&km, k, cs, paged->num_blocks, paged->block_size, s.hkv, s.head_dim, 1, 64, paged->fp8);
    if (!rc) rc = make_map(&vm, v, cs, paged->num_blocks, paged->block_size, s.hkv, s.head_dim, 1, 64, paged->fp8);
  } else {
    rc = make_map(&km, k, ks, s.batch, s.hkv, s.seq_kv, s.head_dim, 64, 1);
    if (!rc) rc = make_map(&vm, v, vs, s.batch, s.hkv, s.seq_kv, s.head_dim, 64, 1);
  }
  if (rc) return rc;
  p.batch = s.batch;
  p.hq = s.hq;
  p.hkv = s.hkv;
  p.group = s.group;
  p.seq_q = s.seq_q;
  p.seq_kv = s.seq_kv;
  p.block_m = pl.block_m;
  p.n_mtiles = pl.n_mtiles;
  p.rows = pl.rows;
  p.nsplit = pl.nsplit;
  p.chunk = pl.chunk;
  cudaError_t e;
  const bool bf = dtype == GQA_DTYPE_BF16;
  if (paged && paged->fp8)
    e = bf ? launch_stream_hd<128, true, true>(p, pl, km, vm, st) : launch_stream_hd<128, false, true>(p, pl, km, vm, st);
  else if (s.head_dim == 128)
    e = bf ? launch_stream_hd<128, true>(p, pl, km, vm, st) : launch_stream_hd<128, false>(p, pl, km, vm, st);
  else
    e = bf ? launch_stream_hd<64, true>(p, pl, km, vm, st) : launch_stream_hd<64, false>(p, pl, km, vm, st);
  return e == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

template <int HD, bool BF, bool SP, bool PG>
cudaError_t launch_prefill_inst(dim3 grid, cudaStream_t st, const PrefillParams& p, const CUtensorMap& qm,
                                const CUtensorMap& km, const CUtensorMap& vm, const CUtensorMap& om) {
  return launch_pdl(gqa_prefill_kernel<HD, BF, SP, PG>, grid, PrefillCfg<HD>::kThreads, PrefillCfg<HD>::kSmemBytes,
                    st, p, qm, km, vm, om);
}

template <int HD, bool BF>
cudaError_t launch_prefill_hd(bool split, bool paged, dim3 grid, cudaStream_t st, const PrefillParams& p,
                              const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                              const CUtensorMap& om) {
  // The unsplit instantiations carry no split code; the dense ones no paging code.
  if (paged)
    return split ? launch_prefill_inst<HD, BF, true, true>(grid, st, p, qm, km, vm, om)
                 : launch_prefill_inst<HD, BF, false, true>(grid, st, p, qm, km, vm, om);
  return split ? launch_prefill_inst<HD, BF, true, false>(grid, st, p, qm, km, vm, om)
               : launch_prefill_inst<HD, BF, false, false>(grid, st, p, qm, km, vm, om);
}

// Launches the tcgen05 prefill kernel for plan `pp` (split dropped when the workspace
// cannot hold the partials). With `paged`, k/v are paged caches, `p` already carries
// the block table and lengths, and s.seq_kv is the bound of the lengths.
int run_prefill(const Shape& s, PrefillPlan pp, const void* q, const void* k, const void* v, void* o,
                const int64_t* qs, const int64_t* ks, const int64_t* vs, const int64_t* os, float scale_log2,
                int causal, int dtype, void* workspace, size_t workspace_bytes, cudaStream_t st,
                const PagedCache* paged = nullptr, PrefillParams p = PrefillParams{}) {
  if (pp.nsplit > 1 &&
      (!workspace || workspace_bytes < prefill_ws_bytes(pp, s.head_dim) || !aligned16(workspace))) {
    pp.nsplit = 1;  // no room for the partials: one CTA per unit
    pp.chunk_tiles = 0;
  }
  p.batch = s.batch;
  p.hq = s.hq;
  p.hkv = s.hkv;
  p.group = s.group;
  p.seq_q = s.seq_q;
  p.seq_kv = s.seq_kv;
  p.bm = pp.bm;
  p.n_pairs = pp.n_pairs;
  p.head_major = pp.head_major;
  p.unit_inner = pp.head_major ? pp.n_pairs : s.batch * s.hkv;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale_log2;
  p.nsplit = pp.nsplit;
  p.chunk_tiles = pp.chunk_tiles;
  if (pp.nsplit > 1) prefill_ws_carve(pp, s.head_dim, workspace, &p);
  CUtensorMap qm, km, vm, om;
  int rc = make_map(&qm, q, qs, s.batch, s.hq, s.seq_q, s.head_dim, p.bm, s.group);
  if (paged) {
    const int64_t cs[4] = {(int64_t)paged->block_size * s.hkv * s.head_dim, (int64_t)s.hkv * s.head_dim,
                           s.head_dim, 1};
    if (!rc) rc = make_map(&km, k, cs, paged->num_blocks, paged->block_size, s.hkv, s.head_dim, 1, 64);
    if (!rc) rc = make_map(&vm, v, cs, paged->num_blocks, paged->block_size, s.hkv, s.head_dim, 1, 64);
  } else {
    if (!rc) rc = make_map(&km, k, ks, s.batch, s.hkv, s.seq_kv, s.head_dim, 128, 1);
    if (!rc) rc = make_map(&vm, v, vs, s.batch, s.hkv, s.seq_kv, s.head_dim, 128, 1);
  }
  if (!rc) rc = make_map(&om, o, os, s.batch, s.hq, s.seq_q, s.head_dim, p.bm, s.group);
  if (rc) return rc;
  const int64_t grid = (int64_t)p.n_pairs * s.batch * s.hkv * p.nsplit;
  if (grid > 0x7fffffff) return GQA_ERR_INVALID_ARG;
  const bool bf = dtype == GQA_DTYPE_BF16;
  const bool split = p.nsplit > 1;
  const dim3 g((unsigned)grid);
  cudaError_t le;
  if (s.head_dim == 128)
    le = bf ? launch_prefill_hd<128, true>(split, paged != nullptr, g, st, p, qm, km, vm, om)
            : launch_prefill_hd<128, false>(split, paged != nullptr, g, st, p, qm, km, vm, om);
  else
    le = bf ? launch_prefill_hd<64, true>(split, paged != nullptr, g, st, p, qm, km, vm, om)
            : launch_prefill_hd<64, false>(split, paged != nullptr, g, st, p, qm, km, vm, om);
  if (le != cudaSuccess) {
    (void)cudaGetLastError();
    return GQA_ERR_CUDA;
  }
  return launch_status();
}

int fill_nan(void* o, const int64_t* os, const Shape& s, int dtype, cudaStream_t st) {
  const int64_t n = (int64_t)s.batch * s.hq * s.seq_q * s.head_dim;
  if (n == 0) return GQA_OK;
  const uint16_t nan_bits = dtype == GQA_DTYPE_BF16 ? 0x7fc0 : 0x7e00;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 4096);
  gqa_fill_nan_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<uint16_t*>(o), os[0], os[1], os[2], s.batch,
                                              s.hq, s.seq_q, s.head_dim, nan_bits);
  return launch_status();
}

int check_common(const void* q, const void* k, const void* v, const int64_t* qs, const int64_t* ks,
                 const int64_t* vs, int dtype) {
  if (dtype != GQA_DTYPE_BF16 && dtype != GQA_DTYPE_F16) return GQA_ERR_UNSUPPORTED;
  int rc = check_strides(q, qs);
  if (!rc) rc = check_strides(k, ks);
  if (!rc) rc = check_strides(v, vs);
  return rc;
}

// Paged forward over 16-bit or (fp8) e4m3 caches; the C ABI's gqa_paged_fwd and
// gqa_paged_fwd_kv8.
int paged_forward(const void* q, const void* k_cache, const void* v_cache, void* o, const int64_t* qs,
                  const int64_t* os, const int* block_table, int bt_stride, const int* seq_lens, int num_seqs,
                  int num_heads, int num_kv_heads, int seq_q, int head_dim, int block_size, int num_blocks,
                  int max_seq_len, float scale_log2, int causal, int dtype, void* workspace, size_t workspace_bytes,
                  void* stream, bool fp8, float k_scale, float v_scale) {
  Shape s;
  int rc = check_shape(num_seqs, num_heads, num_kv_heads, seq_q, max_seq_len, head_dim, &s);
  if (rc) return rc;
  if (!qs || !os) return GQA_ERR_INVALID_ARG;
  if (num_seqs == 0 || seq_q == 0) return GQA_OK;
  if (dtype != GQA_DTYPE_BF16 && dtype != GQA_DTYPE_F16) return GQA_ERR_UNSUPPORTED;
  if (block_size < 64 || (block_size & (block_size - 1)) != 0 || num_blocks <= 0) return GQA_ERR_UNSUPPORTED;
  // fp8 K/V: the streaming kernel only (decode and short chunks), rows of 128 e4m3 values.
  if (fp8 && (head_dim != 128 || !use_stream(s))) return GQA_ERR_UNSUPPORTED;
  if (fp8 && !(k_scale > 0.f && v_scale > 0.f)) return GQA_ERR_INVALID_ARG;
  if (!k_cache || !v_cache || !block_table || !seq_lens || bt_stride <= 0) return GQA_ERR_INVALID_ARG;
  if (max_seq_len > (int64_t)bt_stride * block_size) return GQA_ERR_INVALID_ARG;
  if (!aligned16(k_cache) || !aligned16(v_cache)) return GQA_ERR_ALIGNMENT;
  rc = check_strides(q, qs);
  if (!rc) rc = check_strides(o, os);
  if (rc) return rc;
  int sm = 0;
  rc = current_device(&sm);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (max_seq_len == 0) return fill_nan(o, os, s, dtype, st);
  int shift = 0;
  while ((1 << shift) < block_size) ++shift;
  const PagedCache pc{block_size, num_blocks, fp8};

  if (use_stream(s)) {  // decode and short chunks: the streaming kernel
    StreamPlan pl = plan_stream(s, sm, true);
    StreamParams p{};
    p.q = reinterpret_cast<const uint16_t*>(q);
    p.o = o;
    p.q_sb = qs[0]; p.q_sh = qs[1]; p.q_sm = qs[2];
    p.o_sb = os[0]; p.o_sh = os[1]; p.o_sm = os[2];
    p.causal = causal ? 1 : 0;
    p.scale_log2 = fp8 ? scale_log2 * k_scale : scale_log2;
    p.v_scale = fp8 ? v_scale : 1.0f;
    p.kv_offset = 0;
    p.seq_kv_total = max_seq_len;
    p.block_table = block_table;
    p.seq_lens = seq_lens;
    p.bt_stride = bt_stride;
    p.block_shift = shift;
    if (pl.nsplit > 1 && workspace && workspace_bytes >= stream_ws_bytes(pl, head_dim)) {
      p.mode = kStreamFused;
      stream_ws_carve(pl, head_dim, workspace, &p);
    } else {
      pl = plan_stream(s, sm, false);
      p.mode = kStreamOut;
    }
    return run_stream(s, pl, p, k_cache, v_cache, nullptr, nullptr, dtype, st, &pc);
  }

  PrefillParams p{};  // longer chunks: the tcgen05 prefill kernel over the paged cache
  p.block_table = block_table;
  p.seq_lens = seq_lens;
  p.bt_stride = bt_stride;
  p.block_shift = shift;
  p.num_blocks = num_blocks;
  return run_prefill(s, plan_prefill(s, sm, causal != 0), q, k_cache, v_cache, o, qs, nullptr, nullptr, os,
                     scale_log2, causal, dtype, workspace, workspace_bytes, st, &pc, p);
}

}  // namespace
}  // namespace gqa

using namespace gqa;

extern "C" {

const char* gqa_strerror(int code) {
  switch (code) {
    case GQA_OK: return "success";
    case GQA_ERR_INVALID_ARG: return "invalid argument (shape, null pointer or negative size)";
    case GQA_ERR_UNSUPPORTED: return "unsupported configuration (head_dim 64 or 128, dtype f16/bf16, "
                                     "num_heads/num_kv_heads a power of two <= 128; paged: block_size a power "
                                     "of two >= 64; fp8 K/V: head_dim 128 and group * seq_q <= 64)";
    case GQA_ERR_ALIGNMENT: return "tensor must be contiguous in head_dim with 16-byte aligned base and strides";
    case GQA_ERR_CUDA: return "CUDA runtime or driver call failed";
    case GQA_ERR_TIMEOUT: return "bounded in-kernel wait expired (kernel aborted)";
    case GQA_ERR_WORKSPACE: return "workspace missing or too small";
    case GQA_ERR_NO_DEVICE: return "no sm_100 (B200) device is current";
    case GQA_ERR_SCRATCH_LIMIT: return "problem needs more scratch than the static no-allocation buffer "
                                       "(GQA_NOALLOC_SCRATCH_BYTES) holds";
    case GQA_ERR_DEBUG_CHECK: return "a debug build's in-kernel address or coordinate check failed (access skipped)";
    default: return "unknown gqa status code";
  }
}

int gqa_version(void) { return 100; }

int gqa_sm_count(void) {
  int sm = 0;
  return current_device(&sm) == GQA_OK ? sm : 0;
}

size_t gqa_paged_decode_workspace_bytes(int num_seqs, int num_heads, int num_kv_heads, int max_seq_len,
                                        int head_dim) {
  return gqa_paged_fwd_workspace_bytes(num_seqs, num_heads, num_kv_heads, 1, max_seq_len, head_dim);
}

int gqa_paged_decode(const void* q, const void* k_cache, const void* v_cache, void* o, const int64_t* qs3,
                     const int64_t* os3, const int* block_table, int bt_stride, const int* seq_lens, int num_seqs,
                     int num_heads, int num_kv_heads, int head_dim, int block_size, int num_blocks, int max_seq_len,
                     float scale_log2, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (!qs3 || !os3) return GQA_ERR_INVALID_ARG;
  const int64_t qs[4] = {qs3[0], qs3[1], 0, qs3[2]};  // (b, h, s, d), one query position
  const int64_t os[4] = {os3[0], os3[1], 0, os3[2]};
  // The one new token of each sequence sees all its cached keys.
  return gqa_paged_fwd(q, k_cache, v_cache, o, qs, os, block_table, bt_stride, seq_lens, num_seqs, num_heads,
                       num_kv_heads, 1, head_dim, block_size, num_blocks, max_seq_len, scale_log2, 0, dtype,
                       workspace, workspace_bytes, stream);
}

size_t gqa_paged_fwd_workspace_bytes(int num_seqs, int num_heads, int num_kv_heads, int seq_q, int max_seq_len,
                                     int head_dim) {
  return gqa_fwd_workspace_bytes(num_seqs, num_heads, num_kv_heads, seq_q, max_seq_len, head_dim);
}

int gqa_paged_fwd(const void* q, const void* k_cache, const void* v_cache, void* o, const int64_t* qs,
                  const int64_t* os, const int* block_table, int bt_stride, const int* seq_lens, int num_seqs,
                  int num_heads, int num_kv_heads, int seq_q, int head_dim, int block_size, int num_blocks,
                  int max_seq_len, float scale_log2, int causal, int dtype, void* workspace, size_t workspace_bytes,
                  void* stream) {
  return gqa::paged_forward(q, k_cache, v_cache, o, qs, os, block_table, bt_stride, seq_lens, num_seqs, num_heads,
                            num_kv_heads, seq_q, head_dim, block_size, num_blocks, max_seq_len, scale_log2, causal,
                            dtype, workspace, workspace_bytes, stream, false, 1.0f, 1.0f);
}

int gqa_paged_fwd_kv8(const void* q, const void* k_cache, const void* v_cache, void* o, const int64_t* qs,
                      const int64_t* os, const int* block_table, int bt_stride, const int* seq_lens, int num_seqs,
                      int num_heads, int num_kv_heads, int seq_q, int head_dim, int block_size, int num_blocks,
                      int max_seq_len, float scale_log2, float k_scale, float v_scale, int causal, int dtype,
                      void* workspace, size_t workspace_bytes, void* stream) {
  return gqa::paged_forward(q, k_cache, v_cache, o, qs, os, block_table, bt_stride, seq_lens, num_seqs, num_heads,
                            num_kv_heads, seq_q, head_dim, block_size, num_blocks, max_seq_len, scale_log2, causal,
                            dtype, workspace, workspace_bytes, stream, true, k_scale, v_scale);
}

int gqa_paged_kv_append(const void* key, const void* value, const int64_t* k_strides3, const int64_t* v_strides3,
                        void* k_cache, void* v_cache, const int64_t* slot_mapping, int num_tokens, int num_kv_heads,
                        int head_dim, int block_size, int num_blocks, int dtype, int cache_fp8, float k_scale,
                        float v_scale, void* stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks <= 0) return GQA_ERR_INVALID_ARG;
  if (head_dim != 64 && head_dim != 128) return GQA_ERR_UNSUPPORTED;
  if (dtype != GQA_DTYPE_BF16 && dtype != GQA_DTYPE_F16) return GQA_ERR_UNSUPPORTED;
  if (cache_fp8 && !(k_scale > 0.f && v_scale > 0.f && k_scale < INFINITY && v_scale < INFINITY))
    return GQA_ERR_INVALID_ARG;
  if (num_tokens == 0) return GQA_OK;
  if (!key || !value || !k_strides3 || !v_strides3 || !k_cache || !v_cache || !slot_mapping)
    return GQA_ERR_INVALID_ARG;
  if (!aligned16(key) || !aligned16(value) || !aligned16(k_cache) || !aligned16(v_cache)) return GQA_ERR_ALIGNMENT;
  for (const int64_t* st : {k_strides3, v_strides3}) {
    if (st[2] != 1) return GQA_ERR_ALIGNMENT;
    for (int i = 0; i < 2; ++i)
      if (st[i] < 0 || (st[i] % 8) != 0) return GQA_ERR_ALIGNMENT;
  }
  int sm = 0;
  const int rc = current_device(&sm);
  if (rc) return rc;
  AppendParams p{};
  p.key = reinterpret_cast<const uint16_t*>(key);
  p.value = reinterpret_cast<const uint16_t*>(value);
  p.k_st = k_strides3[0]; p.k_sh = k_strides3[1];
  p.v_st = v_strides3[0]; p.v_sh = v_strides3[1];
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.slot_mapping = slot_mapping;
  p.num_tokens = num_tokens;
  p.hkv = num_kv_heads;
  p.num_slots = (int64_t)num_blocks * block_size;
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  const int64_t rows = (int64_t)num_tokens * num_kv_heads;
  const int blocks = (int)std::min<int64_t>((rows + 7) / 8, (int64_t)sm * 16);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool bf = dtype == GQA_DTYPE_BF16, f8 = cache_fp8 != 0;
#define GQA_APPEND(HD, BF, F8) gqa_kv_append_kernel<HD, BF, F8><<<blocks, 256, 0, st>>>(p)
  if (head_dim == 128) {
    if (f8) { if (bf) GQA_APPEND(128, true, true); else GQA_APPEND(128, false, true); }
    else { if (bf) GQA_APPEND(128, true, false); else GQA_APPEND(128, false, false); }
  } else {
    if (f8) { if (bf) GQA_APPEND(64, true, true); else GQA_APPEND(64, false, true); }
    else { if (bf) GQA_APPEND(64, true, false); else GQA_APPEND(64, false, false); }
  }
#undef GQA_APPEND
  return launch_status();
}

int gqa_prefill_plan(int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv, int head_dim, int causal,
                     int sm_count, int* plan) {
  Shape s;
  const int rc = check_shape(batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim, &s);
  if (rc) return rc;
  if (!plan || sm_count <= 0) return GQA_ERR_INVALID_ARG;
  const PrefillPlan pl = plan_prefill(s, sm_count, causal != 0);
  plan[0] = pl.units;
  plan[1] = pl.nsplit;
  plan[2] = pl.chunk_tiles;
  plan[3] = pl.head_major;
  plan[4] = pl.units * pl.nsplit;
  return GQA_OK;
}

size_t gqa_fwd_workspace_bytes(int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv, int head_dim) {
  Shape s;
  if (check_shape(batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim, &s)) return 0;
  if (seq_q == 0 || seq_kv == 0 || batch == 0) return 0;
  int sm = 0;
  if (current_device(&sm)) return 0;
  if (!use_stream(s)) return prefill_ws_bytes(plan_prefill(s, sm), head_dim);
  const StreamPlan pl = plan_stream(s, sm, true);
  return pl.nsplit > 1 ? stream_ws_bytes(pl, head_dim) : 0;
}

int gqa_fwd(const void* q, const void* k, const void* v, void* o, const int64_t* qs, const int64_t* ks,
            const int64_t* vs, const int64_t* os, int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv,
            int head_dim, float scale_log2, int causal, int dtype, void* workspace, size_t workspace_bytes,
            void* stream) {
  Shape s;
  int rc = check_shape(batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim, &s);
  if (rc) return rc;
  if (batch == 0 || seq_q == 0) return GQA_OK;
  if (dtype != GQA_DTYPE_BF16 && dtype != GQA_DTYPE_F16) return GQA_ERR_UNSUPPORTED;
  rc = check_strides(o, os);
  if (rc) return rc;
  int sm = 0;
  rc = current_device(&sm);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // No key at all (k and v may have no storage): every row sees nothing -> NaN.
  if (seq_kv == 0) return fill_nan(o, os, s, dtype, st);
  rc = check_common(q, k, v, qs, ks, vs, dtype);
  if (rc) return rc;

  if (use_stream(s)) {
    StreamPlan pl = plan_stream(s, sm, true);
    StreamParams p{};
    p.q = reinterpret_cast<const uint16_t*>(q);
    p.o = o;
    p.q_sb = qs[0]; p.q_sh = qs[1]; p.q_sm = qs[2];
    p.o_sb = os[0]; p.o_sh = os[1]; p.o_sm = os[2];
    p.causal = causal ? 1 : 0;
    p.scale_log2 = scale_log2;
    p.kv_offset = 0;
    p.seq_kv_total = seq_kv;
    if (pl.nsplit > 1 && workspace && workspace_bytes >= stream_ws_bytes(pl, head_dim)) {
      p.mode = kStreamFused;
      stream_ws_carve(pl, head_dim, workspace, &p);
    } else {
      pl = plan_stream(s, sm, false);
      p.mode = kStreamOut;
    }
    return run_stream(s, pl, p, k, v, ks, vs, dtype, st);
  }

  // tcgen05 prefill path
  return run_prefill(s, plan_prefill(s, sm, causal != 0), q, k, v, o, qs, ks, vs, os, scale_log2, causal, dtype,
                     workspace, workspace_bytes, st);
}

int gqa_split_first(const void* q, const void* k, const void* v, float* m_p, float* l_p, float* acc_p,
                    const int64_t* qs, const int64_t* ks, const int64_t* vs, const int64_t* ps, const int64_t* as,
                    int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv, int head_dim,
                    float scale_log2, int causal, int splits, int dtype, void* stream) {
  Shape s;
  int rc = check_shape(batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim, &s);
  if (rc) return rc;
  if (splits <= 0 || !m_p || !l_p || !acc_p || !ps || !as) return GQA_ERR_INVALID_ARG;
  if (batch == 0 || seq_q == 0) return GQA_OK;
  if (s.group > kStreamMaxRows) return GQA_ERR_UNSUPPORTED;
  rc = check_common(q, k, v, qs, ks, vs, dtype);
  if (rc) return rc;
  int sm = 0;
  rc = current_device(&sm);
  if (rc) return rc;
  if (seq_kv == 0) return GQA_ERR_INVALID_ARG;
  StreamPlan pl = plan_stream(s, sm, false);
  pl.nsplit = splits;
  pl.chunk = (seq_kv + splits - 1) / splits;  // the reference's chunk size, tl.cdiv(seq_kv, SPLITS)
  StreamParams p{};
  p.q = reinterpret_cast<const uint16_t*>(q);
  p.q_sb = qs[0]; p.q_sh = qs[1]; p.q_sm = qs[2];
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale_log2;
  p.kv_offset = 0;
  p.seq_kv_total = seq_kv;
  p.mode = kStreamRefPartial;
  p.m_p = m_p; p.l_p = l_p; p.acc_p = acc_p;
  p.p_sb = ps[0]; p.p_sh = ps[1]; p.p_sm = ps[2]; p.p_ss = ps[3];
  p.a_sb = as[0]; p.a_sh = as[1]; p.a_sm = as[2]; p.a_ss = as[3]; p.a_sd = as[4];
  if ((int64_t)pl.units * splits > 0x7fffffff) return GQA_ERR_INVALID_ARG;
  return run_stream(s, pl, p, k, v, ks, vs, dtype, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace {
// gqa_split_reduce's checks and launch; `peer` adds the peer exchange's wait
// (counters, epoch, units per source, parity stride) to the combine.
int split_reduce_impl(const float* m_p, const float* l_p, const float* acc_p, void* o, const int64_t* ps,
                      const int64_t* as, const int64_t* os, int batch, int num_heads, int seq_q, int head_dim,
                      int splits, int dtype, void* stream, const CombineParams* peer) {
  if (!m_p || !l_p || !acc_p || !o || !ps || !as || !os) return GQA_ERR_INVALID_ARG;
  if (batch < 0 || num_heads <= 0 || seq_q < 0 || splits <= 0) return GQA_ERR_INVALID_ARG;
  if (head_dim != 64 && head_dim != 128) return GQA_ERR_UNSUPPORTED;
  if (dtype != GQA_DTYPE_BF16 && dtype != GQA_DTYPE_F16) return GQA_ERR_UNSUPPORTED;
  if (os[3] != 1 || (reinterpret_cast<uintptr_t>(o) & 3u)) return GQA_ERR_ALIGNMENT;
  for (int i = 0; i < 3; ++i)
    if (os[i] % 2) return GQA_ERR_ALIGNMENT;
  if (batch == 0 || seq_q == 0) return GQA_OK;
  int rc = current_device(nullptr);
  if (rc) return rc;
  CombineParams p{};
  p.m = m_p; p.l = l_p; p.acc = acc_p; p.o = o;
  p.p_sb = ps[0]; p.p_sh = ps[1]; p.p_sm = ps[2]; p.p_ss = ps[3];
  p.a_sb = as[0]; p.a_sh = as[1]; p.a_sm = as[2]; p.a_ss = as[3]; p.a_sd = as[4];
  p.o_sb = os[0]; p.o_sh = os[1]; p.o_sm = os[2];
  p.batch = batch; p.hq = num_heads; p.seq_q = seq_q; p.head_dim = head_dim; p.nsplit = splits;
  if (peer) {
    p.cnt = peer->cnt;
    p.epoch = peer->epoch;
    p.units = peer->units;
    p.parity_stride = peer->parity_stride;
  }
  const int64_t rows = (int64_t)batch * num_heads * seq_q;
  const int64_t blocks = (rows + 3) / 4;
  if (blocks > 0x7fffffff) return GQA_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == GQA_DTYPE_BF16)
    gqa_combine_kernel<true><<<(unsigned)blocks, 128, 0, st>>>(p);
  else
    gqa_combine_kernel<false><<<(unsigned)blocks, 128, 0, st>>>(p);
  return launch_status();
}
}  // namespace

extern "C" {

int gqa_split_reduce(const float* m_p, const float* l_p, const float* acc_p, void* o, const int64_t* ps,
                     const int64_t* as, const int64_t* os, int batch, int num_heads, int seq_q, int head_dim,
                     int splits, int dtype, void* stream) {
  return split_reduce_impl(m_p, l_p, acc_p, o, ps, as, os, batch, num_heads, seq_q, head_dim, splits, dtype, stream,
                           nullptr);
}

size_t gqa_split_fused_workspace_bytes(int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv,
                                       int head_dim) {
  Shape s;
  if (check_shape(batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim, &s)) return 0;
  if (s.group > kStreamMaxRows || seq_q == 0 || seq_kv == 0 || batch == 0) return 0;
  int sm = 0;
  if (current_device(&sm)) return 0;
  return stream_ws_bytes(plan_stream(s, sm, true), head_dim);
}

int gqa_split_fused(const void* q, const void* k, const void* v, void* o, const int64_t* qs, const int64_t* ks,
                    const int64_t* vs, const int64_t* os, int batch, int num_heads, int num_kv_heads, int seq_q,
                    int seq_kv, int head_dim, float scale_log2, int causal, int dtype, void* workspace,
                    size_t workspace_bytes, void* stream) {
  Shape s;
  int rc = check_shape(batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim, &s);
  if (rc) return rc;
  if (batch == 0 || seq_q == 0) return GQA_OK;
  if (s.group > kStreamMaxRows) return GQA_ERR_UNSUPPORTED;
  if (dtype != GQA_DTYPE_BF16 && dtype != GQA_DTYPE_F16) return GQA_ERR_UNSUPPORTED;
  rc = check_strides(o, os);
  if (rc) return rc;
  int sm = 0;
  rc = current_device(&sm);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (seq_kv == 0) return fill_nan(o, os, s, dtype, st);
  rc = check_common(q, k, v, qs, ks, vs, dtype);
  if (rc) return rc;
  const StreamPlan pl = plan_stream(s, sm, true);
  if (!workspace || workspace_bytes < stream_ws_bytes(pl, head_dim) || !aligned16(workspace))
    return GQA_ERR_WORKSPACE;
  StreamParams p{};
  p.q = reinterpret_cast<const uint16_t*>(q);
  p.o = o;
  p.q_sb = qs[0]; p.q_sh = qs[1]; p.q_sm = qs[2];
  p.o_sb = os[0]; p.o_sh = os[1]; p.o_sm = os[2];
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale_log2;
  p.kv_offset = 0;
  p.seq_kv_total = seq_kv;
  p.mode = kStreamFused;
  stream_ws_carve(pl, head_dim, workspace, &p);
  return run_stream(s, pl, p, k, v, ks, vs, dtype, st);
}

}  // extern "C"

// ----------------------------------------------------------------------------- no-allocation variant
// Scratch of gqa_split_fused_noalloc. Host code must not pass the symbol itself
// to a kernel (in host code it names a host-side stand-in); its device address
// comes from cudaGetSymbolAddress, looked up once per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[GQA_NOALLOC_SCRATCH_BYTES];

namespace gqa {
namespace {
std::vector<void*> g_noalloc_addr;  // per device, guarded by g_mutex

int noalloc_scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GQA_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_mutex);
  if ((int)g_noalloc_addr.size() <= dev) g_noalloc_addr.resize(dev + 1, nullptr);
  if (!g_noalloc_addr[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return GQA_ERR_CUDA;
    g_noalloc_addr[dev] = ptr;
  }
  *out = g_noalloc_addr[dev];
  return GQA_OK;
}
}  // namespace
}  // namespace gqa

extern "C" {

int gqa_split_fused_noalloc(const void* q, const void* k, const void* v, void* o, const int64_t* qs,
                            const int64_t* ks, const int64_t* vs, const int64_t* os, int batch, int num_heads,
                            int num_kv_heads, int seq_q, int seq_kv, int head_dim, float scale_log2, int causal,
                            int dtype, void* stream) {
  Shape s;
  int rc = check_shape(batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim, &s);
  if (rc) return rc;
  if (batch == 0 || seq_q == 0) return GQA_OK;
  if (s.group > kStreamMaxRows) return GQA_ERR_UNSUPPORTED;
  if (dtype != GQA_DTYPE_BF16 && dtype != GQA_DTYPE_F16) return GQA_ERR_UNSUPPORTED;
  rc = check_strides(o, os);
  if (rc) return rc;
  int sm = 0;
  rc = current_device(&sm);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (seq_kv == 0) return fill_nan(o, os, s, dtype, st);
  rc = check_common(q, k, v, qs, ks, vs, dtype);
  if (rc) return rc;
  const StreamPlan pl = plan_stream(s, sm, true);
  if (stream_ws_bytes(pl, head_dim) > (size_t)GQA_NOALLOC_SCRATCH_BYTES) return GQA_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  rc = noalloc_scratch_address(&scratch);
  if (rc) return rc;
  StreamParams p{};
  p.q = reinterpret_cast<const uint16_t*>(q);
  p.o = o;
  p.q_sb = qs[0]; p.q_sh = qs[1]; p.q_sm = qs[2];
  p.o_sb = os[0]; p.o_sh = os[1]; p.o_sm = os[2];
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale_log2;
  p.kv_offset = 0;
  p.seq_kv_total = seq_kv;
  p.mode = kStreamFused;
  stream_ws_carve(pl, head_dim, scratch, &p);
  // The array keeps the previous call's contents, possibly laid out for another
  // shape: the ticket counters must read zero, so clear them on this stream.
  if (cudaMemsetAsync(p.ws_cnt, 0, (size_t)pl.units * sizeof(unsigned), st) != cudaSuccess) return GQA_ERR_CUDA;
  return run_stream(s, pl, p, k, v, ks, vs, dtype, st);
}

size_t gqa_partial_workspace_bytes(int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv_local,
                                   int head_dim) {
  Shape s;
  if (check_shape(batch, num_heads, num_kv_heads, seq_q, seq_kv_local, head_dim, &s)) return 0;
  if (s.group > kStreamMaxRows || seq_q == 0 || batch == 0) return 0;
  int sm = 0;
  if (current_device(&sm)) return 0;
  return stream_ws_bytes(plan_stream(s, sm, true), head_dim);
}

}  // extern "C"

namespace {
// The peer-exchange outputs of gqa_partial_peer (nullptr: gqa_partial's own arrays).
struct PeerArgs {
  float* const* bases;
  unsigned long long* const* cnts;
  int npeer, rank;
  const unsigned long long* epoch;
  int64_t slot, parity;
};

int partial_impl(const void* q, const void* k, const void* v, float* m_out, float* l_out, float* acc_out,
                 const int64_t* qs, const int64_t* ks, const int64_t* vs, int batch, int num_heads, int num_kv_heads,
                 int seq_q, int seq_kv_local, int kv_offset, int seq_kv_total, int head_dim, float scale_log2,
                 int causal, int dtype, void* workspace, size_t workspace_bytes, void* stream, const PeerArgs* peer) {
  Shape s;
  int rc = check_shape(batch, num_heads, num_kv_heads, seq_q, seq_kv_local, head_dim, &s);
  if (rc) return rc;
  if (!peer && (!m_out || !l_out || !acc_out)) return GQA_ERR_INVALID_ARG;
  if (kv_offset < 0 || seq_kv_total < kv_offset + seq_kv_local) return GQA_ERR_INVALID_ARG;
  if (batch == 0 || seq_q == 0) return GQA_OK;
  if (s.group > kStreamMaxRows) return GQA_ERR_UNSUPPORTED;
  if (dtype != GQA_DTYPE_BF16 && dtype != GQA_DTYPE_F16) return GQA_ERR_UNSUPPORTED;
  if (!peer && !aligned16(acc_out)) return GQA_ERR_ALIGNMENT;
  int sm = 0;
  rc = current_device(&sm);
  if (rc) return rc;
  if (peer && seq_kv_local == 0) return GQA_ERR_UNSUPPORTED;  // every rank must hold keys
  if (seq_kv_local == 0) {
    // An empty shard (more ranks than 64-key blocks) is a valid part: (-inf, 0, 0)
    // for every row, which the combine weighs 0. k and v may have no storage.
    const int64_t rows = (int64_t)batch * num_heads * seq_q;
    const int blocks = (int)std::min<int64_t>((rows * head_dim + 255) / 256, 4096);
    gqa_fill_empty_partial_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(m_out, l_out, acc_out,
                                                                                           rows, head_dim);
    return launch_status();
  }
  rc = check_common(q, k, v, qs, ks, vs, dtype);
  if (rc) return rc;
  const StreamPlan pl = plan_stream(s, sm, true);
  if (!workspace || workspace_bytes < stream_ws_bytes(pl, head_dim) || !aligned16(workspace))
    return GQA_ERR_WORKSPACE;
  StreamParams p{};
  p.q = reinterpret_cast<const uint16_t*>(q);
  p.q_sb = qs[0]; p.q_sh = qs[1]; p.q_sm = qs[2];
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale_log2;
  p.kv_offset = kv_offset;
  p.seq_kv_total = seq_kv_total;
  p.mode = kStreamFusedPartial;
  p.m_out = m_out; p.l_out = l_out; p.acc_out = acc_out;
  if (peer) {
    const int64_t rows = (int64_t)batch * num_heads * seq_q;
    p.npeer = peer->npeer;
    p.my_rank = peer->rank;
    for (int i = 0; i < peer->npeer; ++i) {
      p.peer_base[i] = peer->bases[i];
      p.peer_cnt[i] = peer->cnts[i];
    }
    p.epoch = peer->epoch;
    p.peer_slot = peer->slot;
    p.peer_parity = peer->parity;
    p.pk_rows = rows;
    p.pk_acc = (2 * rows + 3) / 4 * 4;
  }
  stream_ws_carve(pl, head_dim, workspace, &p);
  return run_stream(s, pl, p, k, v, ks, vs, dtype, reinterpret_cast<cudaStream_t>(stream));
}
}  // namespace

extern "C" {

int gqa_partial(const void* q, const void* k, const void* v, float* m_out, float* l_out, float* acc_out,
                const int64_t* qs, const int64_t* ks, const int64_t* vs, int batch, int num_heads, int num_kv_heads,
                int seq_q, int seq_kv_local, int kv_offset, int seq_kv_total, int head_dim, float scale_log2,
                int causal, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  return partial_impl(q, k, v, m_out, l_out, acc_out, qs, ks, vs, batch, num_heads, num_kv_heads, seq_q, seq_kv_local,
                      kv_offset, seq_kv_total, head_dim, scale_log2, causal, dtype, workspace, workspace_bytes, stream,
                      nullptr);
}

int gqa_lse_combine(const float* m_parts, const float* l_parts, const float* acc_parts, int nparts,
                    int64_t ml_part_stride, int64_t acc_part_stride, void* o, const int64_t* os, int batch,
                    int num_heads, int seq_q, int head_dim, int dtype, void* stream) {
  if (nparts <= 0 || batch < 0 || seq_q < 0 || num_heads <= 0) return GQA_ERR_INVALID_ARG;
  if (ml_part_stride < 0 || acc_part_stride < 0) return GQA_ERR_INVALID_ARG;
  const int64_t ps[4] = {(int64_t)num_heads * seq_q, (int64_t)seq_q, 1, ml_part_stride};
  const int64_t as[5] = {(int64_t)num_heads * seq_q * head_dim, (int64_t)seq_q * head_dim, (int64_t)head_dim,
                         acc_part_stride, 1};
  return gqa_split_reduce(m_parts, l_parts, acc_parts, o, ps, as, os, batch, num_heads, seq_q, head_dim, nparts,
                          dtype, stream);
}

// ---- peer exchange (key-sharded multi-GPU combine without a collective library)
static_assert(sizeof(cudaIpcMemHandle_t) == GQA_IPC_HANDLE_BYTES, "IPC handle size");

int gqa_exchange_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return GQA_ERR_INVALID_ARG;
  int rc = current_device(nullptr);
  if (rc) return rc;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return GQA_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return GQA_ERR_CUDA;
  }
  *ptr = p;
  return GQA_OK;
}

int gqa_exchange_free(void* ptr) { return (!ptr || cudaFree(ptr) == cudaSuccess) ? GQA_OK : GQA_ERR_CUDA; }

int gqa_ipc_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return GQA_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) return GQA_ERR_CUDA;
  std::memcpy(handle, &h, sizeof(h));
  return GQA_OK;
}

int gqa_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return GQA_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return GQA_ERR_CUDA;
  return GQA_OK;
}

int gqa_ipc_close(void* ptr) { return (ptr && cudaIpcCloseMemHandle(ptr) == cudaSuccess) ? GQA_OK : GQA_ERR_CUDA; }

int gqa_epoch_bump(unsigned long long* epoch, void* stream) {
  if (!epoch) return GQA_ERR_INVALID_ARG;
  gqa_epoch_bump_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(epoch);
  return launch_status();
}

int gqa_partial_units(int batch, int num_heads, int num_kv_heads, int seq_q, int head_dim, int* units) {
  if (!units) return GQA_ERR_INVALID_ARG;
  Shape s;
  const int rc = check_shape(batch, num_heads, num_kv_heads, seq_q, 1, head_dim, &s);
  if (rc) return rc;
  *units = (batch == 0 || seq_q == 0) ? 0 : plan_stream(s, 1, false).units;
  return GQA_OK;
}

int gqa_partial_peer(const void* q, const void* k, const void* v, const int64_t* qs, const int64_t* ks,
                     const int64_t* vs, int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv_local,
                     int kv_offset, int seq_kv_total, int head_dim, float scale_log2, int causal, int dtype,
                     float* const* peer_bases, unsigned long long* const* peer_cnts, int npeer, int rank,
                     const unsigned long long* epoch, int64_t slot_floats, int64_t parity_floats, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (!peer_bases || !peer_cnts || !epoch || npeer < 1 || npeer > kMaxPeers || rank < 0 || rank >= npeer)
    return GQA_ERR_INVALID_ARG;
  const int64_t rows = (int64_t)batch * num_heads * seq_q;
  const int64_t packed = (2 * rows + 3) / 4 * 4 + rows * head_dim;
  if (slot_floats < packed || parity_floats < npeer * slot_floats) return GQA_ERR_INVALID_ARG;
  if (slot_floats % 4 || parity_floats % 4) return GQA_ERR_ALIGNMENT;
  for (int i = 0; i < npeer; ++i) {
    if (!peer_bases[i] || !peer_cnts[i]) return GQA_ERR_INVALID_ARG;
    if (!aligned16(peer_bases[i]) || (reinterpret_cast<uintptr_t>(peer_cnts[i]) & 7u)) return GQA_ERR_ALIGNMENT;
  }
  const PeerArgs pa{peer_bases, peer_cnts, npeer, rank, epoch, slot_floats, parity_floats};
  return partial_impl(q, k, v, nullptr, nullptr, nullptr, qs, ks, vs, batch, num_heads, num_kv_heads, seq_q,
                      seq_kv_local, kv_offset, seq_kv_total, head_dim, scale_log2, causal, dtype, workspace,
                      workspace_bytes, stream, &pa);
}

int gqa_lse_combine_peer(const float* recv, const unsigned long long* cnt, const unsigned long long* epoch,
                         int nparts, int64_t slot_floats, int64_t parity_floats, int units, void* o, const int64_t* os,
                         int batch, int num_heads, int seq_q, int head_dim, int dtype, void* stream) {
  if (!recv || !cnt || !epoch || nparts < 1 || nparts > kMaxPeers || units < 1) return GQA_ERR_INVALID_ARG;
  if (batch < 0 || seq_q < 0 || num_heads <= 0 || slot_floats < 0 || parity_floats < nparts * slot_floats)
    return GQA_ERR_INVALID_ARG;
  const int64_t rows = (int64_t)batch * num_heads * seq_q;
  const int64_t acc_off = (2 * rows + 3) / 4 * 4;
  const int64_t ps[4] = {(int64_t)num_heads * seq_q, (int64_t)seq_q, 1, slot_floats};
  const int64_t as[5] = {(int64_t)num_heads * seq_q * head_dim, (int64_t)seq_q * head_dim, (int64_t)head_dim,
                         slot_floats, 1};
  CombineParams peer{};
  peer.cnt = cnt;
  peer.epoch = epoch;
  peer.units = (unsigned long long)units;
  peer.parity_stride = parity_floats;
  return split_reduce_impl(recv, recv + rows, recv + acc_off, o, ps, as, os, batch, num_heads, seq_q, head_dim, nparts,
                           dtype, stream, &peer);
}

#ifdef GQA_DEBUG_CHECKS
namespace gqa {
__global__ void gqa_exp2_poly2_kernel(const float* x, float* y, int n) {
  const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i + 1 < n) {
    const float2 r = exp2_poly2(make_float2(x[i], x[i + 1]));
    y[i] = r.x;
    y[i + 1] = r.y;
  } else if (i < n) {
    y[i] = exp2_poly2(make_float2(x[i], x[i])).x;
  }
}
}  // namespace gqa
#endif

int gqa_debug_inject(int cta, int load, long long wait_limit_ns) {
#ifdef GQA_DEBUG_CHECKS
  const int rc = current_device(nullptr);
  if (rc) return rc;
  const unsigned long long lim = wait_limit_ns > 0 ? (unsigned long long)wait_limit_ns : kWaitLimitNs;
  if (cudaMemcpyToSymbol(g_withhold_cta, &cta, sizeof(int)) != cudaSuccess) return GQA_ERR_CUDA;
  if (cudaMemcpyToSymbol(g_withhold_load, &load, sizeof(int)) != cudaSuccess) return GQA_ERR_CUDA;
  if (cudaMemcpyToSymbol(g_wait_limit_ns, &lim, sizeof(lim)) != cudaSuccess) return GQA_ERR_CUDA;
  return GQA_OK;
#else
  (void)cta; (void)load; (void)wait_limit_ns;
  return GQA_ERR_UNSUPPORTED;
#endif
}

int gqa_debug_exp2_poly2(const float* x, float* y, int n, void* stream) {
#ifdef GQA_DEBUG_CHECKS
  if (!x || !y || n < 0) return GQA_ERR_INVALID_ARG;
  const int rc = current_device(nullptr);
  if (rc) return rc;
  if (n == 0) return GQA_OK;
  const int threads = 256, pairs = (n + 1) / 2;
  gqa_exp2_poly2_kernel<<<(pairs + threads - 1) / threads, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, y, n);
  return launch_status();
#else
  (void)x; (void)y; (void)n; (void)stream;
  return GQA_ERR_UNSUPPORTED;
#endif
}

int gqa_device_error(int* code, int* site, int clear) {
  int rc = current_device(nullptr);
  if (rc) return rc;
  int c = 0, s = 0;
  if (cudaMemcpyFromSymbol(&c, g_device_error, sizeof(int)) != cudaSuccess) return GQA_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&s, g_device_error_site, sizeof(int)) != cudaSuccess) return GQA_ERR_CUDA;
  if (code) *code = c;
  if (site) *site = s;
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return GQA_ERR_CUDA;
    if (cudaMemcpyToSymbol(g_device_error_site, &zero, sizeof(int)) != cudaSuccess) return GQA_ERR_CUDA;
  }
  return GQA_OK;
}

}  // extern "C"
