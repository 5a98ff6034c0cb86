// pt_api.cu -- C ABI of the library (declared in include/pathtile_b200.h):
// argument checks, tile planning, TMA descriptor encoding and launches.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "pathtile_b200.h"
#define PT_KERNELS_IMPL 1
#include "pt_cl.h"
#include "pt_frozen_config.h"
#include "pt_kernels.cuh"
#include "pt_peer.cuh"
#include "pt_registry.h"
#include "pt_tc.h"

// Device error word (one per device context); kernels receive its address.
__device__ unsigned int g_pt_device_error;

namespace {

constexpr int kMaxDevices = 64;
constexpr int kGenericRows = 128;

thread_local int t_last_cuda_error = 0;
// Device whose primary context this host thread has made current.  Driver
// calls such as cuTensorMapEncodeTiled need a current context, which a fresh
// thread (autograd's backward worker, a data-loader thread) does not have
// until some runtime call binds it.
thread_local int t_bound_device = -1;

struct DeviceInfo {
  bool ready = false;
  int sm_count = 0;
  int major = 0;
  int minor = 0;
  int max_smem = 0;  // opt-in dynamic shared memory per block
  unsigned* err = nullptr;
  std::unordered_map<const void*, size_t> smem_attr;  // max dynamic smem already granted
  std::unordered_map<const void*, int> regs;          // registers per thread of a function
};

std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];
std::once_flag g_once;
std::vector<pt::Entry>* g_entries = nullptr;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
// Rows are padded to a bank-conflict-free pitch by a TMA box wider than the
// row; if the driver ever rejects such a box, rows fall back to pitch L.
bool g_padded_box_ok = true;
// Launch options: a configuration and an engine per path, each either set or
// left to the frozen table.  g_opts holds the process-wide overrides
// (pt_set_config / pt_set_engine); the *_ex entry points make their caller's
// options current on this host thread for the duration of the call, so two
// callers with different options never see each other's choices.
struct Opts {
  pt::LaunchCfg cfg[3] = {};
  bool has_cfg[3] = {false, false, false};
  int engine[3] = {-1, -1, -1};  // -1: the frozen table decides
  int bwd_kernel = -1;           // PT_BWD_*; -1: the frozen table decides
  int helper_channels = -1;      // -1: the frozen table decides
};
Opts g_opts;
thread_local const Opts* t_opts = nullptr;

const Opts& opts() { return t_opts ? *t_opts : g_opts; }

// Makes `o` the current options of this host thread until the scope ends.
struct OptsScope {
  const Opts* saved;
  explicit OptsScope(const Opts* o) : saved(t_opts) {
    if (o) t_opts = o;
  }
  ~OptsScope() { t_opts = saved; }
};

int cuda_fail(cudaError_t e) {
  t_last_cuda_error = static_cast<int>(e);
  return PT_ERR_CUDA;
}

void init_once() {
  g_entries = new std::vector<pt::Entry>();
  pt::register_shard_0(*g_entries);
  pt::register_shard_1(*g_entries);
  pt::register_shard_2(*g_entries);
  pt::register_shard_3(*g_entries);
  pt::register_shard_4(*g_entries);
  pt::register_shard_5(*g_entries);
  pt::register_shard_6(*g_entries);
  pt::register_shard_7(*g_entries);
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess) {
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  (void)cudaGetLastError();
}

// Current device's info; PT_ERR_DEVICE unless it is compute capability 10.0.
int current_device(DeviceInfo*& di) {
  std::call_once(g_once, init_once);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return PT_ERR_DEVICE;
  if (t_bound_device != dev) {
    if ((e = cudaSetDevice(dev)) != cudaSuccess) return cuda_fail(e);  // binds the primary context
    t_bound_device = dev;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    if ((e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return cuda_fail(e);
    if ((e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
      return cuda_fail(e);
    if ((e = cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
      return cuda_fail(e);
    if ((e = cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) !=
        cudaSuccess)
      return cuda_fail(e);
    if (d.major == 10 && d.minor == 0) {
      void* p = nullptr;
      if ((e = cudaGetSymbolAddress(&p, g_pt_device_error)) != cudaSuccess) return cuda_fail(e);
      d.err = static_cast<unsigned*>(p);
    }
    d.ready = true;
  }
  if (d.major != 10 || d.minor != 0) return PT_ERR_DEVICE;
  di = &d;
  return PT_OK;
}

int ensure_smem_attr(DeviceInfo& di, const void* func, size_t bytes) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = di.smem_attr.find(func);
  if (it != di.smem_attr.end() && it->second >= bytes) return PT_OK;
  cudaError_t e =
      cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess) return cuda_fail(e);
  di.smem_attr[func] = bytes;
  return PT_OK;
}

// Arithmetic-intensity class of a shape (in-range FMAs per output element:
// < 12 light, < 24 medium, else heavy), the key of the frozen table.
int intensity_class(int L, int K) {
  const int pad = K / 2;
  long long pairs = 0;
  for (int j = 0; j < K; ++j) {
    const int lo = pad - j > 0 ? pad - j : 0;
    const int hi = L + pad - j < L ? L + pad - j : L;
    if (hi > lo) pairs += hi - lo;
  }
  if (pairs < 12LL * L) return 0;
  if (pairs < 24LL * L) return 1;
  return 2;
}

pt::LaunchCfg cfg_for(int path, int L, int K) {
  const Opts& o = opts();
  return o.has_cfg[path] ? o.cfg[path] : pt::kFrozenCfg[path][intensity_class(L, K)];
}

int gcd_int(int a, int b) {
  while (b) {
    const int r = a % b;
    a = b;
    b = r;
  }
  return a;
}

// Grid of the tensor-core kernel.  Tiles are dealt round-robin, so CTA g visits
// channels (g + i*G) mod H with period P = H / gcd(G, H).  Take the largest G
// up to min(SMs, tiles) with P <= 2 (the CTA's one or two Toeplitz operands
// then stay resident) as long as it keeps >= 3/4 of that many SMs busy;
// otherwise every SM, with a per-tile rebuild (period 0).
void tensor_grid(int H, long long tiles, int sm_count, int& G, int& period) {
  const int gmax = static_cast<int>(tiles < sm_count ? tiles : sm_count);
  for (int c = gmax; c >= 1 && 4LL * c >= 3LL * gmax; --c) {
    const int P = H / gcd_int(c, H);
    if (P <= 2) {
      G = c;
      period = P;
      return;
    }
  }
  G = gmax;
  period = 0;
}

// Channel groups (super-rows of Hc channels) of the tensor-core kernel.
int tensor_groups(int H, int L) {
  const int hc = pt::tc::layout_for(L).hc;
  return (H + hc - 1) / hc;
}

// Tiles of the tensor-core kernels: 128 batch rows (FWD/DX) or 64 (dK) of one group.
int tensor_rows(int path) { return path == PT_PATH_DK ? pt::tc::kDkRowsPerTile : pt::tc::kRowsPerTile; }

long long tensor_tiles(int path, int B, int groups) {
  const int r = tensor_rows(path);
  return static_cast<long long>((B + r - 1) / r) * groups;
}

// Engine of a path at a shape: PT_ENGINE_TENSOR (tcgen05, L % 4 == 0 and a TMA
// encoder) or PT_ENGINE_FFMA (CUDA-core kernels, every shape).  Shapes without
// a specialised CUDA-core kernel take the tensor engine where it applies.  The frozen
// table's tensor choice applies only to full tiles (48 % L == 0: one
// 48-column channel or 48 / L packed channels per tile row; partially filled
// tiles measured faster on the FFMA kernels) and needs a grid in which every
// CTA visits at most two channel groups; an explicit pt_set_engine override
// needs neither for FWD/DX (they rebuild the Toeplitz operand per tile
// otherwise), while dK always needs its accumulators resident.
const pt::Entry* find_entry(int L, int K);

int engine_for(int path, int B, int H, int L, int K, int sm_count) {
  if (L % 4 != 0 || g_encode == nullptr) return PT_ENGINE_FFMA;
  const int groups = tensor_groups(H, L);
  int G = 0, period = 0;
  tensor_grid(groups, tensor_tiles(path, B, groups), sm_count > 0 ? sm_count : 148, G, period);
  const int forced = opts().engine[path];
  if (forced >= 0) {
    if (path == PT_PATH_DK && period == 0) return PT_ENGINE_FFMA;
    return forced;
  }
  // The frozen table compares the tensor engine with the specialised CUDA-core
  // kernels; a shape without one would run the generic kernels (runtime bounds,
  // many times slower), so it takes the tensor engine wherever that applies.
  if (find_entry(L, K) == nullptr) {
    if (path == PT_PATH_DK) return period > 0 ? PT_ENGINE_TENSOR : PT_ENGINE_FFMA;
    return PT_ENGINE_TENSOR;
  }
  if (48 % L != 0 || pt::kFrozenEngine[path][intensity_class(L, K)] != PT_ENGINE_TENSOR)
    return PT_ENGINE_FFMA;
  return period > 0 ? PT_ENGINE_TENSOR : PT_ENGINE_FFMA;
}

const pt::Entry* find_entry(int L, int K) {
  for (const pt::Entry& e : *g_entries)
    if (e.L == L && e.K == K) return &e;
  return nullptr;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int round_up(int v, int q) { return (v + q - 1) / q * q; }

struct Plan {
  bool exact = false;
  bool tensor = false;  // tcgen05 FWD/DX kernel (grid g.G)
  int period = 0;       // tensor kernel: channel groups per CTA (1, 2), or 0 for per-tile Toeplitz rebuilds
  int groups = 0;       // tensor kernel: channel groups of hc channels
  pt::tc::Layout lay{1, 3, false};
  int loader = 0;
  const void* func = nullptr;
  pt::TileGeom g{};
  int threads = 0;
  size_t smem = 0;
  pt::tc::BwdSched sched{};  // fused backward: work schedule
};

// Row pitch (floats) for TMA3D tiles: 128-bit LDS by 8 consecutive rows hits
// 8 distinct 16-byte bank groups iff pitch/4 is odd.
int tma_pitch(int L) { return (!g_padded_box_ok || (L / 4) % 2 == 1) ? L : L + 4; }

// Internal path id of plan_exact: the fused CUDA-core backward (bwd_rows_kernel),
// planned with the dK path's launch configuration and one thread per row.
constexpr int kPathBwdRows = 4;

int plan_exact(int path, int B, int H, int L, int K, DeviceInfo& di, const pt::Entry& e, Plan& p) {
  const bool bwd = (path == kPathBwdRows);
  const bool two_inputs = bwd || path == PT_PATH_DK;
  const pt::LaunchCfg cfg = cfg_for(bwd ? PT_PATH_DK : path, L, K);
  pt::TileGeom& g = p.g;
  g.B = B;
  g.H = H;
  g.L = L;
  g.K = K;
  // Tile shape: every channel in one block whenever H fits a TMA box (<= 256),
  // with as many batches as reach `rows`; above that, balanced channel blocks
  // of at most `rows` channels (a multiple of 4 so 1-D bulk tiles stay
  // 16-byte aligned), so no block is left mostly idle.
  const int R = cfg.rows;
  if (H <= 256) {
    g.Th = H;
    g.Tb = R / H;
    if (g.Tb < 1) g.Tb = 1;
    g.nhb = 1;
  } else {
    const int nb = (H + R - 1) / R;
    g.Th = ((H + nb - 1) / nb + 3) / 4 * 4;
    g.Tb = 1;
    g.nhb = (H + g.Th - 1) / g.Th;
  }
  g.Q = (B + g.Tb - 1) / g.Tb;
  g.stages = cfg.stages;
  p.loader = e.loader;
  g.pitch = (e.loader == pt::LOAD_TMA3D) ? tma_pitch(L) : L;
  const int T = g.Th * g.Tb;
  const long long tile_bytes = static_cast<long long>(g.pitch) * T * 4;
  long long stage = (tile_bytes + 1023) / 1024 * 1024;
  // Buffers: DK and the fused backward = (dy, x) per stage; FWD/DX = one in-place buffer per stage.
  auto n_buf = [&](int stages) { return two_inputs ? 2 * stages : stages; };
  // mbarriers: full + done per stage (+ the fused backward's stores-done barrier, padded to 16 bytes).
  auto bars = [&](int stages) { return 2LL * stages * 8 + (bwd ? 16 : 0); };
  // Fewer stages when the buffers would not fit the per-block shared memory.
  while (g.stages > 2 && static_cast<long long>(n_buf(g.stages)) * stage + bars(g.stages) + 1024 > di.max_smem)
    --g.stages;
  if (two_inputs) {
    // The idle ring doubles as the [K][T] in-CTA reduction buffer at the end.
    const long long red = static_cast<long long>(K) * T * 4;
    if (n_buf(g.stages) * stage < red)
      stage = ((red + n_buf(g.stages) - 1) / n_buf(g.stages) + 1023) / 1024 * 1024;
  }
  const long long bar_bytes = bars(g.stages);
  if (static_cast<long long>(n_buf(g.stages)) * stage + bar_bytes + 1024 > di.max_smem)
    return PT_ERR_UNSUPPORTED;
  g.stage_bytes = static_cast<unsigned>(stage);
  g.tx_bytes = static_cast<unsigned>(tile_bytes);
  p.smem = static_cast<size_t>(n_buf(g.stages)) * stage + static_cast<size_t>(bar_bytes) + 1024;
  // Two consumer threads per row only while the CTA stays within 288 threads
  // (the kernels' launch bound); larger tiles run one thread per row.
  const int tpr = (!bwd && cfg.tpr == 2 && 2 * round_up(T, 32) + 32 <= 288) ? 2 : 1;
  p.threads = tpr * round_up(T, 32) + 32;  // consumer warps (tpr per row) + one producer warp
  p.func = bwd                    ? e.bwd
           : (path == PT_PATH_FWD) ? e.fwd[tpr - 1]
           : (path == PT_PATH_DX)  ? e.dx[tpr - 1]
                                   : e.dk[tpr - 1];
  p.exact = true;
  int rc = ensure_smem_attr(di, p.func, p.smem);
  if (rc != PT_OK) return rc;
  int occ = 0;
  cudaError_t ce = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, p.func, p.threads, p.smem);
  if (ce != cudaSuccess) return cuda_fail(ce);
  if (occ < 1) return PT_ERR_UNSUPPORTED;
  const int cps = cfg.ctas_per_sm < occ ? cfg.ctas_per_sm : occ;
  long long G = static_cast<long long>(di.sm_count) * cps;
  const long long tiles = static_cast<long long>(g.Q) * g.nhb;
  if (G > tiles) G = tiles;
  G = G / g.nhb * g.nhb;
  if (G < g.nhb) G = g.nhb;
  g.G = static_cast<int>(G);
  return PT_OK;
}

// Bucketed generic kernels (compile-time maxima 16 / 32 / 48 for L and K).
int bucket48(int n) { return n <= 16 ? 16 : (n <= 32 ? 32 : 48); }

template <int OP>
const void* conv_bucket_func(int L, int K) {
  const int lm = bucket48(L), km = bucket48(K);
#define PT_CB(LM, KM) \
  if (lm == LM && km == KM) return reinterpret_cast<const void*>(&pt::conv_bucket_kernel<LM, KM, OP>);
  PT_CB(16, 16) PT_CB(16, 32) PT_CB(16, 48) PT_CB(32, 16) PT_CB(32, 32) PT_CB(32, 48)
  PT_CB(48, 16) PT_CB(48, 32) PT_CB(48, 48)
#undef PT_CB
  return nullptr;
}

const void* dk_bucket_func(int L, int K) {
  const int lm = bucket48(L), km = bucket48(K);
#define PT_DB(LM, KM) \
  if (lm == LM && km == KM) return reinterpret_cast<const void*>(&pt::dk_bucket_kernel<LM, KM>);
  PT_DB(16, 16) PT_DB(16, 32) PT_DB(16, 48) PT_DB(32, 16) PT_DB(32, 32) PT_DB(32, 48)
  PT_DB(48, 16) PT_DB(48, 32) PT_DB(48, 48)
#undef PT_DB
  return nullptr;
}

void plan_generic_dk(int B, int H, int L, int K, const DeviceInfo& di, Plan& p) {
  pt::TileGeom& g = p.g;
  g.B = B;
  g.H = H;
  g.L = L;
  g.K = K;
  g.Th = H;
  g.Tb = 1;
  g.nhb = 1;
  // One wave of CTAs at the bucketed kernel's occupancy.
  int per_sm = 0;
  const void* f = dk_bucket_func(L, K);
  if (!f || cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, f, 128, 0) != cudaSuccess || per_sm < 1)
    per_sm = 2;
  int G = di.sm_count * per_sm;
  if (G > B) G = B;
  if (G < 1) G = 1;
  g.G = G;
  p.exact = false;
}

int plan_tensor(int path, int B, int H, int L, int K, DeviceInfo& di, Plan& p) {
  pt::TileGeom& g = p.g;
  g.B = B;
  g.H = H;
  g.L = L;
  g.K = K;
  p.lay = pt::tc::layout_for(L);
  p.func = (path == PT_PATH_DK) ? pt::tc::dk_func(p.lay) : pt::tc::conv_func(path, p.lay);
  p.smem = (path == PT_PATH_DK) ? pt::tc::dk_smem(p.lay) : pt::tc::conv_smem(p.lay);
  p.threads = (path == PT_PATH_DK) ? pt::tc::kDkThreads : pt::tc::kThreads;
  if (!p.func || static_cast<long long>(p.smem) > di.max_smem) return PT_ERR_UNSUPPORTED;
  int rc = ensure_smem_attr(di, p.func, p.smem);
  if (rc != PT_OK) return rc;
  p.groups = tensor_groups(H, L);
  const long long tiles = tensor_tiles(path, B, p.groups);
  g.Q = static_cast<int>(tiles);  // tiles of 128 (64 for dK) batch rows of one channel group
  tensor_grid(p.groups, tiles, di.sm_count, g.G, p.period);
  if (path == PT_PATH_DK && p.period == 0) return PT_ERR_UNSUPPORTED;
  g.Th = 1;
  g.Tb = tensor_rows(path);
  g.nhb = H;
  p.exact = true;
  p.tensor = true;
  return PT_OK;
}

int plan(int path, int B, int H, int L, int K, DeviceInfo& di, Plan& p) {
  if (engine_for(path, B, H, L, K, di.sm_count) == PT_ENGINE_TENSOR)
    return plan_tensor(path, B, H, L, K, di, p);
  const pt::Entry* e = find_entry(L, K);
  const bool tma_ok = g_encode != nullptr;
  if (e && ((e->loader == pt::LOAD_TMA3D && tma_ok) ||
            (e->loader == pt::LOAD_BULK1D && (static_cast<long long>(H) * L) % 4 == 0)))
    return plan_exact(path, B, H, L, K, di, *e, p);
  if (path == PT_PATH_DK) plan_generic_dk(B, H, L, K, di, p);
  p.exact = false;
  return PT_OK;
}

// 3-D tensor map over a [B,H,L] float tensor with box (pitch, Th, Tb).
int encode_rows_tmap(CUtensorMap* tm, const float* base, const pt::TileGeom& g) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(g.L), static_cast<cuuint64_t>(g.H),
                        static_cast<cuuint64_t>(g.B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(g.L) * 4,
                           static_cast<cuuint64_t>(g.L) * g.H * 4};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(g.pitch), static_cast<cuuint32_t>(g.Th),
                       static_cast<cuuint32_t>(g.Tb)};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims,
                        strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = static_cast<int>(r);
    return PT_ERR_CUDA;
  }
  return PT_OK;
}

// Encode the two tensor maps of a TMA3D plan.  If the driver refuses the
// padded-pitch box, switch every later plan to pitch L, re-plan and retry.
int encode_pair(int path, int B, int H, int L, int K, DeviceInfo& di, Plan& p, CUtensorMap* a,
                const float* pa, CUtensorMap* b, const float* pb) {
  int rc = encode_rows_tmap(a, pa, p.g);
  if (rc == PT_OK) rc = encode_rows_tmap(b, pb, p.g);
  if (rc == PT_OK || p.g.pitch == L) return rc;
  g_padded_box_ok = false;
  if (path == kPathBwdRows) {
    const pt::Entry* e = find_entry(L, K);
    if (!e || (rc = plan_exact(path, B, H, L, K, di, *e, p)) != PT_OK) return e ? rc : PT_ERR_UNSUPPORTED;
  } else if ((rc = plan(path, B, H, L, K, di, p)) != PT_OK) {
    return rc;
  }
  rc = encode_rows_tmap(a, pa, p.g);
  if (rc == PT_OK) rc = encode_rows_tmap(b, pb, p.g);
  return rc;
}

// Tensor map of the tensor-core path: box of `cols` floats x 128 batch rows
// with the 128-B (cols 32) or 64-B (cols 16) swizzle; 3-D over (L, H, B) with
// one channel per box, or 2-D over [B, H*L] for packed super-rows.
int encode_tc_tmap(CUtensorMap* tm, const float* base, int B, int H, int L, int cols, bool packed,
                   int rows = pt::tc::kRowsPerTile, bool atom32 = false) {
  cuuint64_t dims3[3] = {static_cast<cuuint64_t>(L), static_cast<cuuint64_t>(H),
                         static_cast<cuuint64_t>(B)};
  cuuint64_t strides3[2] = {static_cast<cuuint64_t>(L) * 4, static_cast<cuuint64_t>(L) * H * 4};
  cuuint32_t box3[3] = {static_cast<cuuint32_t>(cols), 1u, static_cast<cuuint32_t>(rows)};
  cuuint64_t dims2[2] = {static_cast<cuuint64_t>(L) * H, static_cast<cuuint64_t>(B)};
  cuuint64_t strides2[1] = {static_cast<cuuint64_t>(L) * H * 4};
  cuuint32_t box2[2] = {static_cast<cuuint32_t>(cols), static_cast<cuuint32_t>(rows)};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, packed ? 2 : 3, const_cast<float*>(base),
                        packed ? dims2 : dims3, packed ? strides2 : strides3, packed ? box2 : box3, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                               : (cols == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B),
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = static_cast<int>(r);
    return PT_ERR_CUDA;
  }
  return PT_OK;
}

int launch_tensor(const Plan& p, const float* in, const float* taps, float* out, unsigned* err,
                  cudaStream_t stream) {
  const pt::TileGeom& g = p.g;
  const int lb = p.lay.lb;
  const bool packed = p.lay.packed;
  CUtensorMap in128, in64, out128, out64;
  std::memset(&in128, 0, sizeof(in128));
  std::memset(&in64, 0, sizeof(in64));
  std::memset(&out128, 0, sizeof(out128));
  std::memset(&out64, 0, sizeof(out64));
  int rc = PT_OK;
  if (lb >= 2) {
    if ((rc = encode_tc_tmap(&in128, in, g.B, g.H, g.L, 32, packed)) != PT_OK) return rc;
    if ((rc = encode_tc_tmap(&out128, out, g.B, g.H, g.L, 32, packed)) != PT_OK) return rc;
  }
  if (lb & 1) {
    if ((rc = encode_tc_tmap(&in64, in, g.B, g.H, g.L, 16, packed)) != PT_OK) return rc;
    if ((rc = encode_tc_tmap(&out64, out, g.B, g.H, g.L, 16, packed)) != PT_OK) return rc;
  }
  int H = g.H, L = g.L, K = g.K, hc = p.lay.hc, groups = p.groups, n_tiles = g.Q, period = p.period;
  void* args[] = {&in128, &in64, &out128, &out64, const_cast<float**>(&taps), &H, &L, &K, &hc,
                  &groups, &n_tiles, &period, &err};
  const cudaError_t ce = cudaLaunchKernel(p.func, dim3(g.G), dim3(p.threads), args, p.smem, stream);
  if (ce != cudaSuccess) return cuda_fail(ce);
  return PT_OK;
}

// Workspace of the tensor-core dK: per CTA and resident group, Hc*K partials,
// then the group id of each (CTA, slot).
size_t tensor_dk_ws_bytes(const Plan& p) {
  const size_t slots = static_cast<size_t>(p.g.G) * pt::tc::kDkMaxGroups;
  const size_t part = (slots * p.lay.hc * p.g.K * sizeof(float) + 255) / 256 * 256;
  return part + slots * sizeof(int);
}

int launch_tensor_dk(const Plan& p, const float* dy, const float* x, float* dk, int mode, void* ws,
                     unsigned* err, cudaStream_t stream) {
  const pt::TileGeom& g = p.g;
  const bool packed = p.lay.packed;
  const int rows = pt::tc::kDkRowsPerTile;
  const int lb = p.lay.lb;
  CUtensorMap dy128, dy64, x32b;
  std::memset(&dy128, 0, sizeof(dy128));
  std::memset(&dy64, 0, sizeof(dy64));
  std::memset(&x32b, 0, sizeof(x32b));
  int rc = PT_OK;
  if (lb >= 2 && (rc = encode_tc_tmap(&dy128, dy, g.B, g.H, g.L, 32, packed, rows)) != PT_OK) return rc;
  if ((lb & 1) && (rc = encode_tc_tmap(&dy64, dy, g.B, g.H, g.L, 16, packed, rows)) != PT_OK) return rc;
  // x feeds the MMAs as an MN-major tf32 operand: 32-column boxes, 128-B swizzle of 32-B atoms.
  if ((rc = encode_tc_tmap(&x32b, x, g.B, g.H, g.L, 32, packed, rows, true)) != PT_OK) return rc;
  const int atomic = (mode == PT_DK_ATOMIC) ? 1 : 0;
  float* out = atomic ? dk : static_cast<float*>(ws);
  const size_t slots = static_cast<size_t>(g.G) * pt::tc::kDkMaxGroups;
  const size_t part_bytes = (slots * p.lay.hc * g.K * sizeof(float) + 255) / 256 * 256;
  int* group_of = atomic ? nullptr : reinterpret_cast<int*>(static_cast<unsigned char*>(ws) + part_bytes);
  int H = g.H, L = g.L, K = g.K, hc = p.lay.hc, groups = p.groups, n_tiles = g.Q, period = p.period;
  void* args[] = {&dy128, &dy64, &x32b, &out, &group_of, &H, &L, &K, &hc, &groups, &n_tiles, &period,
                  const_cast<int*>(&atomic), &err};
  cudaError_t ce = cudaLaunchKernel(p.func, dim3(g.G), dim3(p.threads), args, p.smem, stream);
  if (ce != cudaSuccess) return cuda_fail(ce);
  if (!atomic) {
    pt::tc::dk_reduce(out, group_of, static_cast<int>(slots), H, K, hc, dk,
                      mode == PT_DK_DETERMINISTIC_ACCUMULATE ? 1 : 0, stream);
    if ((ce = cudaGetLastError()) != cudaSuccess) return cuda_fail(ce);
  }
  return PT_OK;
}

// pt_dx_dk's kernel choice at a shape: the caller's, else the frozen table's.
pt::BwdChoice bwd_choice(int L, int K) {
  const Opts& o = opts();
  pt::BwdChoice c = pt::kFrozenBwd[intensity_class(L, K)];
  if (o.bwd_kernel >= 0) c.kernel = o.bwd_kernel;
  if (o.helper_channels >= 0) c.helper_channels = o.helper_channels;
  return c;
}

// Work schedule of the tensor-core fused backward on `sms` SMs (pt::tc::BwdSched):
// kp = floor(min(tiles, sms) / H) primary CTAs per channel; the E = sms - kp*H
// SMs left over become helpers that take every channel's tail blocks when that
// shortens the busiest CTA by at least 3 % (a helper's channel switch counted
// as one tile; P chosen to balance primaries and helpers) and no helper owns
// more than max_helper_channels channels (the frozen per-class limit, or the
// caller's).  Otherwise the plain grid of kp*H
// CTAs, which must keep at least 3/4 of min(tiles, SMs) busy.  A channel switch
// drains the helper's MMA pipeline while the Toeplitz operand is rebuilt (the
// shared memory holds one), so many switches cost more than the extra SMs
// give: measured at B = 16384, L = K = 48, helpers made H = 64 (4 channels per
// helper) 7 % faster and H = 96 (2 per helper; no plain grid) 24 % faster than
// the separate kernels, but H = 128 (7 per helper) 6 % slower than the plain
// grid, and 11 % slower at K = 3; the frozen table holds the limit per class.
// Returns the grid size, or 0 where the kernel does not apply.
int fused_schedule(int B, int H, int sms, int max_helper_channels, pt::tc::BwdSched& sc) {
  const int nblk = (B + pt::tc::kRowsPerTile - 1) / pt::tc::kRowsPerTile;
  const long long tiles = static_cast<long long>(nblk) * H;
  const int gmax = static_cast<int>(tiles < sms ? tiles : sms);
  const int kp = gmax / H;
  if (kp < 1) return 0;
  const int plain = (nblk + kp - 1) / kp;  // tiles of the busiest CTA in the plain grid
  const int E = sms - kp * H;
  int best_cost = plain, best_p = 0;
  if (E >= 1 && nblk >= 2 && (H + E - 1) / E <= max_helper_channels) {
    const int m = (H + E - 1) / E;
    for (int P = 1; P < nblk; ++P) {
      const int prim = (P + kp - 1) / kp;
      const int help = m * (nblk - P) + (m - 1);
      const int cost = prim > help ? prim : help;
      if (cost < best_cost) {
        best_cost = cost;
        best_p = P;
      }
    }
    if (best_p > 0 && 100LL * best_cost <= 97LL * plain) {
      sc = pt::tc::BwdSched{H, nblk, kp, best_p, E, m, 0};
      return sms;
    }
  }
  const int G = kp * H;
  if (4LL * G < 3LL * gmax) return 0;
  sc = pt::tc::BwdSched{H, nblk, kp, nblk, 0, 0, kp == 1 ? 1 : 0};
  return G;
}

// Fused backward (dX on the tensor cores, dK on the CUDA cores, one pass over dy
// and x): rows of 32 < L <= 48 columns with L % 4 == 0 and any K <= 48 (the
// kernel's 48-column layout), dX not forced onto the CUDA cores, and a schedule
// from fused_schedule.
bool plan_fused(int B, int H, int L, int K, DeviceInfo& di, Plan& p) {
  const void* func = pt::tc::bwd_func(L, K);
  if (!func || g_encode == nullptr) return false;
  const int dx_engine = opts().engine[PT_PATH_DX];
  if (dx_engine >= 0 && dx_engine != PT_ENGINE_TENSOR) return false;
  if (static_cast<long long>(pt::tc::bwd_smem()) > di.max_smem) return false;
  pt::tc::BwdSched sc{};
  const int G = fused_schedule(B, H, di.sm_count, bwd_choice(L, K).helper_channels, sc);
  if (G < 1) return false;
  if (ensure_smem_attr(di, func, pt::tc::bwd_smem()) != PT_OK) return false;
  // The kernel rebalances registers between its warpgroups (setmaxnreg), which
  // draws on the registers the CTA is launched with: launch it only with the
  // per-thread count its split assumes.
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = di.regs.find(func);
    if (it == di.regs.end()) {
      cudaFuncAttributes fa;
      const int regs = (cudaFuncGetAttributes(&fa, func) == cudaSuccess) ? fa.numRegs : 0;
      (void)cudaGetLastError();
      it = di.regs.emplace(func, regs).first;
    }
    if (it->second != pt::tc::kBwdLaunchRegs) return false;
  }
  pt::TileGeom& g = p.g;
  g.B = B;
  g.H = H;
  g.L = L;
  g.K = K;
  g.Q = sc.nblk * H;
  g.G = G;
  g.Th = 1;
  g.Tb = pt::tc::kRowsPerTile;
  g.nhb = H;
  p.func = func;
  p.smem = pt::tc::bwd_smem();
  p.threads = pt::tc::bwd_threads();
  p.exact = true;
  p.tensor = true;
  p.period = 1;
  p.groups = H;
  p.lay = pt::tc::layout_for(L);
  p.sched = sc;
  return true;
}

// Workspace of the fused backward: none in direct mode, else [slots][4][K] partials.
size_t fused_ws_bytes(const Plan& p) {
  const pt::tc::BwdSched& sc = p.sched;
  if (sc.direct) return 0;
  const size_t slots = static_cast<size_t>(sc.kp) * sc.H + static_cast<size_t>(sc.E) * sc.m;
  return (slots * 4 * p.g.K * sizeof(float) + 255) / 256 * 256;
}

int launch_fused(const Plan& p, const float* dy, const float* x, const float* k, float* dx, float* dk,
                 int mode, void* ws, unsigned* err, cudaStream_t stream, const pt::PeerArgs* peers = nullptr) {
  const pt::TileGeom& g = p.g;
  CUtensorMap dy128, dy64, x128, x64, dx128, dx64;
  int rc = PT_OK;
  if ((rc = encode_tc_tmap(&dy128, dy, g.B, g.H, g.L, 32, false)) != PT_OK) return rc;
  if ((rc = encode_tc_tmap(&dy64, dy, g.B, g.H, g.L, 16, false)) != PT_OK) return rc;
  if ((rc = encode_tc_tmap(&x128, x, g.B, g.H, g.L, 32, false)) != PT_OK) return rc;
  if ((rc = encode_tc_tmap(&x64, x, g.B, g.H, g.L, 16, false)) != PT_OK) return rc;
  if ((rc = encode_tc_tmap(&dx128, dx, g.B, g.H, g.L, 32, false)) != PT_OK) return rc;
  if ((rc = encode_tc_tmap(&dx64, dx, g.B, g.H, g.L, 16, false)) != PT_OK) return rc;
  pt::tc::BwdSched sc = p.sched;
  int accumulate = (mode == PT_DK_DETERMINISTIC) ? 0 : 1;  // atomic and *_ACCUMULATE add to dk
  float* part = sc.direct ? nullptr : static_cast<float*>(ws);
  int acc_k = sc.direct ? accumulate : 0;
  pt::PeerArgs pa{};
  pa.world = 1;
  if (peers && sc.direct) pa = *peers;
  void* args[] = {&dy128, &dy64, &x128, &x64, &dx128, &dx64, const_cast<float**>(&k), &part, &dk,
                  &sc, &acc_k, &pa, &err};
  cudaError_t ce = cudaLaunchKernel(p.func, dim3(g.G), dim3(p.threads), args, p.smem, stream);
  if (ce != cudaSuccess) return cuda_fail(ce);
  if (!sc.direct) {
    pt::tc::bwd_dk_reduce(part, dk, sc, g.K, accumulate, stream);
    if ((ce = cudaGetLastError()) != cudaSuccess) return cuda_fail(ce);
  }
  return PT_OK;
}

size_t dk_ws_bytes(const Plan& p);

// Fused backward on the CUDA cores (bwd_rows_kernel): shapes with a specialised
// CUDA-core kernel whose loader applies, where the tensor-core fused kernel
// does not, and where neither dX nor dK is forced onto the tensor cores.  A
// heavy shape (>= 24 in-range FMAs per output) whose separate dX would run on
// the tensor cores stays separate: one thread doing both FMA nests of a row is
// FMA-bound there (measured at B = 16384, H = 96, L = K = 48: 0.348 ms fused on
// the CUDA cores against 0.253 ms for tensor-core dX + CUDA-core dK), while on
// light and medium shapes the saved [B, H, L] stream wins (9-31 % on the edge
// and tuning shapes).
bool plan_bwd_rows(int B, int H, int L, int K, DeviceInfo& di, Plan& p) {
  const Opts& o = opts();
  if (o.engine[PT_PATH_DX] == PT_ENGINE_TENSOR || o.engine[PT_PATH_DK] == PT_ENGINE_TENSOR) return false;
  if (bwd_choice(L, K).kernel == PT_BWD_ANY_FUSED && intensity_class(L, K) == 2 &&
      engine_for(PT_PATH_DX, B, H, L, K, di.sm_count) == PT_ENGINE_TENSOR)
    return false;
  const pt::Entry* e = find_entry(L, K);
  if (!e) return false;
  if (!((e->loader == pt::LOAD_TMA3D && g_encode != nullptr) ||
        (e->loader == pt::LOAD_BULK1D && (static_cast<long long>(H) * L) % 4 == 0)))
    return false;
  return plan_exact(kPathBwdRows, B, H, L, K, di, *e, p) == PT_OK;
}

// The kernel pt_dx_dk runs at a shape (filling p): 1 the tensor-core fused
// kernel, 2 the CUDA-core fused kernel, 0 pt_dx then pt_dk.
int plan_backward(int B, int H, int L, int K, DeviceInfo& di, Plan& p) {
  const int kind = bwd_choice(L, K).kernel;
  if ((kind == PT_BWD_TENSOR_FUSED || kind == PT_BWD_ANY_FUSED) && plan_fused(B, H, L, K, di, p)) return 1;
  if ((kind == PT_BWD_FFMA_FUSED || kind == PT_BWD_ANY_FUSED) && plan_bwd_rows(B, H, L, K, di, p)) return 2;
  return 0;
}

int launch_bwd_rows(Plan& p, DeviceInfo& di, const float* dy, const float* x, const float* k, float* dx,
                    float* dk, int mode, void* ws, size_t ws_bytes, cudaStream_t stream) {
  const int B = p.g.B, H = p.g.H, L = p.g.L, K = p.g.K;
  CUtensorMap tm_dy, tm_x, tm_dx;
  std::memset(&tm_dy, 0, sizeof(tm_dy));
  std::memset(&tm_x, 0, sizeof(tm_x));
  std::memset(&tm_dx, 0, sizeof(tm_dx));
  int rc = PT_OK;
  if (p.loader == pt::LOAD_TMA3D) {
    if ((rc = encode_pair(kPathBwdRows, B, H, L, K, di, p, &tm_dy, dy, &tm_x, x)) != PT_OK) return rc;
    if ((rc = encode_rows_tmap(&tm_dx, dx, p.g)) != PT_OK) return rc;
  }
  const int atomic_mode = (mode == PT_DK_ATOMIC) ? 1 : 0;
  float* dst = dk;
  if (!atomic_mode) {
    if (!ws || ws_bytes < dk_ws_bytes(p)) return PT_ERR_WORKSPACE;
    if (!aligned16(ws)) return PT_ERR_ALIGN;
    dst = static_cast<float*>(ws);
  }
  pt::TileGeom g = p.g;
  unsigned* err = di.err;
  void* args[] = {&tm_dy, &tm_x, &tm_dx, const_cast<float**>(&dy), const_cast<float**>(&x),
                  const_cast<float**>(&k), &dx, &dst, &g, const_cast<int*>(&atomic_mode), &err};
  cudaError_t ce = cudaLaunchKernel(p.func, dim3(g.G), dim3(p.threads), args, p.smem, stream);
  if (ce != cudaSuccess) return cuda_fail(ce);
  if (!atomic_mode) {
    const dim3 grid2((H + 31) / 32, K);
    pt::dk_reduce_kernel<<<grid2, 256, 0, stream>>>(dst, dk, g, mode == PT_DK_DETERMINISTIC_ACCUMULATE ? 1 : 0);
    if ((ce = cudaGetLastError()) != cudaSuccess) return cuda_fail(ce);
  }
  return PT_OK;
}

// act1/act2 are [B,H,L] activations (may be null when B == 0, as an empty
// tensor has no storage); hk is the [H,K] filter or filter gradient.
int check_common(const void* act1, const void* act2, const void* hk, int B, int H, int L, int K) {
  if (B < 0 || H < 1 || L < 1 || K < 1) return PT_ERR_ARGS;
  if (!hk || (B > 0 && (!act1 || !act2))) return PT_ERR_ARGS;
  if (L > PT_MAX_L || K > PT_MAX_K) return PT_ERR_UNSUPPORTED;
  if (static_cast<long long>(B) * H > (1ll << 31)) return PT_ERR_ARGS;
  if (!aligned16(act1) || !aligned16(act2) || !aligned16(hk)) return PT_ERR_ALIGN;
  return PT_OK;
}

int launch_rows(int path, const float* in, const float* taps, float* out, int B, int H, int L, int K,
                cudaStream_t stream) {
  int rc = check_common(in, out, taps, B, H, L, K);
  if (rc != PT_OK) return rc;
  if (B == 0) return PT_OK;
  DeviceInfo* di = nullptr;
  if ((rc = current_device(di)) != PT_OK) return rc;
  Plan p;
  if ((rc = plan(path, B, H, L, K, *di, p)) != PT_OK) return rc;
  cudaError_t ce;
  if (p.tensor) return launch_tensor(p, in, taps, out, di->err, stream);
  if (p.exact) {
    CUtensorMap tm_in, tm_out;
    std::memset(&tm_in, 0, sizeof(tm_in));
    std::memset(&tm_out, 0, sizeof(tm_out));
    if (p.loader == pt::LOAD_TMA3D) {
      if ((rc = encode_pair(path, B, H, L, K, *di, p, &tm_in, in, &tm_out, out)) != PT_OK) return rc;
    }
    unsigned* err = di->err;
    pt::TileGeom g = p.g;
    void* args[] = {&tm_in, &tm_out, const_cast<float**>(&in), const_cast<float**>(&taps), &out, &g, &err};
    ce = cudaLaunchKernel(p.func, dim3(g.G), dim3(p.threads), args, p.smem, stream);
  } else {
    const long long S = static_cast<long long>(B) * H;
    const long long n_tiles = (S + kGenericRows - 1) / kGenericRows;
    long long grid = static_cast<long long>(di->sm_count) * 8;
    if (grid > n_tiles) grid = n_tiles;
    const void* f = (path == PT_PATH_FWD) ? conv_bucket_func<pt::OP_FWD>(L, K) : conv_bucket_func<pt::OP_DX>(L, K);
    if (!f) return PT_ERR_UNSUPPORTED;
    long long nt = n_tiles;
    void* args[] = {const_cast<float**>(&in), const_cast<float**>(&taps), &out, &B, &H, &L, &K, &nt};
    ce = cudaLaunchKernel(f, dim3(static_cast<unsigned>(grid)), dim3(kGenericRows), args, 0, stream);
  }
  if (ce != cudaSuccess) return cuda_fail(ce);
  return PT_OK;
}

bool cfg_valid(int rows_per_tile, int stages, int ctas_per_sm, int threads_per_row) {
  if (rows_per_tile < 32 || rows_per_tile > 256 || rows_per_tile % 32 != 0) return false;
  if (stages < 2 || stages > 4 || ctas_per_sm < 1 || ctas_per_sm > 4) return false;
  return threads_per_row == 1 || threads_per_row == 2;
}

// Validated copy of a caller's per-call options (null: nothing to copy).
bool to_opts(const pt_launch_opts* o, Opts& out) {
  if (!o) return true;
  if (o->bwd_kernel < PT_BWD_FROZEN || o->bwd_kernel > PT_BWD_ANY_FUSED) return false;
  if (o->helper_channels < -1 || o->helper_channels > 1024) return false;
  out.bwd_kernel = o->bwd_kernel;
  out.helper_channels = o->helper_channels;
  for (int p = 0; p < 3; ++p) {
    if (o->engine[p] != -1 && o->engine[p] != PT_ENGINE_FFMA && o->engine[p] != PT_ENGINE_TENSOR) return false;
    out.engine[p] = o->engine[p];
    if (o->rows_per_tile[p] == 0) continue;
    if (!cfg_valid(o->rows_per_tile[p], o->stages[p], o->ctas_per_sm[p], o->threads_per_row[p])) return false;
    out.cfg[p] = pt::LaunchCfg{o->rows_per_tile[p], o->stages[p], o->ctas_per_sm[p], o->threads_per_row[p]};
    out.has_cfg[p] = true;
  }
  return true;
}

// Self-test of the wait limit: warp 0 waits on an mbarrier that nothing arrives
// on, through the same bounded wait as every pipeline kernel but with a short
// limit; the wait runs out, sets DEVERR_TIMEOUT_FULL and the kernel returns.
// Lane 0 records how long the wait lasted and whether it reported success.
__global__ void wait_selftest_kernel(unsigned long long limit_ns, unsigned long long* out, unsigned* err) {
  __shared__ __align__(8) unsigned long long bar;
  const uint32_t b = pt::smem_u32(&bar);
  if (threadIdx.x == 0) {
    pt::mbar_init(b, 1);
    pt::fence_mbar_init();
  }
  __syncthreads();
  const unsigned long long t0 = pt::globaltimer_ns();
  const bool ok = pt::mbar_wait_bounded_for(b, 0, err, pt::DEVERR_TIMEOUT_FULL, limit_ns);
  const unsigned long long t1 = pt::globaltimer_ns();
  if (threadIdx.x == 0) {
    out[0] = t1 - t0;
    out[1] = ok ? 1ull : 0ull;
  }
}

size_t dk_ws_bytes(const Plan& p) {
  return static_cast<size_t>(p.g.G) * p.g.K * p.g.Th * sizeof(float);
}

}  // namespace

extern "C" {

int pt_fwd(const float* x, const float* k, float* y, int B, int H, int L, int K, void* stream) {
  return launch_rows(PT_PATH_FWD, x, k, y, B, H, L, K, static_cast<cudaStream_t>(stream));
}

int pt_dx(const float* dy, const float* k, float* dx, int B, int H, int L, int K, void* stream) {
  return launch_rows(PT_PATH_DX, dy, k, dx, B, H, L, K, static_cast<cudaStream_t>(stream));
}

size_t pt_dk_workspace_bytes(int B, int H, int L, int K) {
  if (B < 1 || H < 1 || L < 1 || K < 1 || L > PT_MAX_L || K > PT_MAX_K) return 0;
  DeviceInfo* di = nullptr;
  if (current_device(di) != PT_OK) return 0;
  Plan p;
  if (plan(PT_PATH_DK, B, H, L, K, *di, p) != PT_OK) return 0;
  return p.tensor ? tensor_dk_ws_bytes(p) : dk_ws_bytes(p);
}

int pt_dk(const float* dy, const float* x, float* dk, int B, int H, int L, int K, int mode, void* ws,
          size_t ws_bytes, void* stream_v) {
  int rc = check_common(dy, x, dk, B, H, L, K);
  if (rc != PT_OK) return rc;
  if (mode != PT_DK_ATOMIC && mode != PT_DK_DETERMINISTIC && mode != PT_DK_DETERMINISTIC_ACCUMULATE)
    return PT_ERR_ARGS;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  cudaError_t ce;
  if (B == 0) {
    if (mode == PT_DK_DETERMINISTIC) {
      ce = cudaMemsetAsync(dk, 0, static_cast<size_t>(H) * K * sizeof(float), stream);
      if (ce != cudaSuccess) return cuda_fail(ce);
    }
    return PT_OK;
  }
  DeviceInfo* di = nullptr;
  if ((rc = current_device(di)) != PT_OK) return rc;
  Plan p;
  if ((rc = plan(PT_PATH_DK, B, H, L, K, *di, p)) != PT_OK) return rc;
  const int atomic_mode = (mode == PT_DK_ATOMIC) ? 1 : 0;
  if (p.tensor) {
    if (!atomic_mode) {
      if (!ws || ws_bytes < tensor_dk_ws_bytes(p)) return PT_ERR_WORKSPACE;
      if (!aligned16(ws)) return PT_ERR_ALIGN;
    }
    return launch_tensor_dk(p, dy, x, dk, mode, ws, di->err, stream);
  }
  float* dst = dk;
  if (!atomic_mode) {
    if (!ws || ws_bytes < dk_ws_bytes(p)) return PT_ERR_WORKSPACE;
    if (!aligned16(ws)) return PT_ERR_ALIGN;
    dst = static_cast<float*>(ws);
  }
  pt::TileGeom g = p.g;
  if (p.exact) {
    CUtensorMap tm_dy, tm_x;
    std::memset(&tm_dy, 0, sizeof(tm_dy));
    std::memset(&tm_x, 0, sizeof(tm_x));
    if (p.loader == pt::LOAD_TMA3D) {
      if ((rc = encode_pair(PT_PATH_DK, B, H, L, K, *di, p, &tm_dy, dy, &tm_x, x)) != PT_OK) return rc;
      if (!atomic_mode && ws_bytes < dk_ws_bytes(p)) return PT_ERR_WORKSPACE;
      g = p.g;
    }
    unsigned* err = di->err;
    void* args[] = {&tm_dy, &tm_x, const_cast<float**>(&dy), const_cast<float**>(&x), &dst, &g,
                    const_cast<int*>(&atomic_mode), &err};
    ce = cudaLaunchKernel(p.func, dim3(g.G), dim3(p.threads), args, p.smem, stream);
  } else {
    const void* f = dk_bucket_func(L, K);
    if (!f) return PT_ERR_UNSUPPORTED;
    int gG = g.G, am = atomic_mode;
    void* args[] = {const_cast<float**>(&dy), const_cast<float**>(&x), &dst, &B, &H, &L, &K, &gG, &am};
    ce = cudaLaunchKernel(f, dim3(g.G), dim3(128), args, 0, stream);
  }
  if (ce != cudaSuccess) return cuda_fail(ce);
  if (!atomic_mode) {
    const dim3 grid2((H + 31) / 32, K);
    pt::dk_reduce_kernel<<<grid2, 256, 0, stream>>>(dst, dk, g,
                                                    mode == PT_DK_DETERMINISTIC_ACCUMULATE ? 1 : 0);
    ce = cudaGetLastError();
    if (ce != cudaSuccess) return cuda_fail(ce);
  }
  return PT_OK;
}

int pt_dx_dk_fused(int B, int H, int L, int K) {
  if (B < 1 || H < 1 || L < 1 || K < 1 || L > PT_MAX_L || K > PT_MAX_K) return 0;
  DeviceInfo* di = nullptr;
  if (current_device(di) != PT_OK) return 0;
  Plan p;
  return plan_backward(B, H, L, K, *di, p);
}

size_t pt_dx_dk_workspace_bytes(int B, int H, int L, int K) {
  if (B < 1 || H < 1 || L < 1 || K < 1 || L > PT_MAX_L || K > PT_MAX_K) return 0;
  DeviceInfo* di = nullptr;
  if (current_device(di) != PT_OK) return 0;
  Plan p;
  const int kind = plan_backward(B, H, L, K, *di, p);
  if (kind == 1) return fused_ws_bytes(p);
  if (kind == 2) return dk_ws_bytes(p);
  return pt_dk_workspace_bytes(B, H, L, K);
}

int pt_dx_dk(const float* dy, const float* x, const float* k, float* dx, float* dk, int B, int H, int L,
             int K, int mode, void* ws, size_t ws_bytes, void* stream_v) {
  int rc = check_common(dy, x, k, B, H, L, K);
  if (rc != PT_OK) return rc;
  if (!dk || (B > 0 && !dx)) return PT_ERR_ARGS;
  if (!aligned16(dx) || !aligned16(dk)) return PT_ERR_ALIGN;
  if (mode != PT_DK_ATOMIC && mode != PT_DK_DETERMINISTIC && mode != PT_DK_DETERMINISTIC_ACCUMULATE)
    return PT_ERR_ARGS;
  if (B == 0) return pt_dk(dy, x, dk, B, H, L, K, mode, ws, ws_bytes, stream_v);
  DeviceInfo* di = nullptr;
  if ((rc = current_device(di)) != PT_OK) return rc;
  Plan p;
  const int kind = plan_backward(B, H, L, K, *di, p);
  if (kind == 1) {
    const size_t need = fused_ws_bytes(p);
    if (need > 0) {
      if (!ws || ws_bytes < need) return PT_ERR_WORKSPACE;
      if (!aligned16(ws)) return PT_ERR_ALIGN;
    }
    return launch_fused(p, dy, x, k, dx, dk, mode, ws, di->err, static_cast<cudaStream_t>(stream_v));
  }
  if (kind == 2)
    return launch_bwd_rows(p, *di, dy, x, k, dx, dk, mode, ws, ws_bytes, static_cast<cudaStream_t>(stream_v));
  if ((rc = pt_dx(dy, k, dx, B, H, L, K, stream_v)) != PT_OK) return rc;
  return pt_dk(dy, x, dk, B, H, L, K, mode, ws, ws_bytes, stream_v);
}

// ---------------- channels-last [B, L, H] ----------------
namespace {

int check_cl(const void* a1, const void* a2, const void* hk, int B, int L, int H, int K) {
  if (B < 0 || H < 1 || L < 1 || K < 1) return PT_ERR_ARGS;
  if (L > PT_MAX_L || K > PT_MAX_K) return PT_ERR_UNSUPPORTED;
  if (!hk || (B > 0 && (!a1 || !a2))) return PT_ERR_ARGS;
  auto al4 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; };
  if (!al4(a1) || !al4(a2) || !al4(hk)) return PT_ERR_ALIGN;
  return PT_OK;
}

int conv_cl(const float* in, const float* k, float* out, int B, int L, int H, int K, bool rev, void* stream) {
  int rc = check_cl(in, out, k, B, L, H, K);
  if (rc != PT_OK || B == 0) return rc;
  DeviceInfo* di = nullptr;
  if ((rc = current_device(di)) != PT_OK) return rc;
  cudaError_t ce = pt::cl::launch_conv(in, k, out, B, L, H, K, rev, static_cast<cudaStream_t>(stream));
  return ce == cudaSuccess ? PT_OK : cuda_fail(ce);
}

}  // namespace

int pt_fwd_cl(const float* x, const float* k, float* y, int B, int L, int H, int K, void* stream) {
  return conv_cl(x, k, y, B, L, H, K, false, stream);
}

int pt_dx_cl(const float* dy, const float* k, float* dx, int B, int L, int H, int K, void* stream) {
  return conv_cl(dy, k, dx, B, L, H, K, true, stream);
}

size_t pt_dk_cl_workspace_bytes(int B, int L, int H, int K) {
  if (B < 1 || H < 1 || L < 1 || K < 1 || L > PT_MAX_L || K > PT_MAX_K) return 0;
  DeviceInfo* di = nullptr;
  if (current_device(di) != PT_OK) return 0;
  return pt::cl::dk_workspace_bytes(B, L, H, K, di->sm_count);
}

int pt_dk_cl(const float* dy, const float* x, float* dk, int B, int L, int H, int K, int accumulate, void* ws,
             size_t ws_bytes, void* stream_v) {
  int rc = check_cl(dy, x, dk, B, L, H, K);
  if (rc != PT_OK) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (B == 0) {
    if (accumulate) return PT_OK;
    cudaError_t ce = cudaMemsetAsync(dk, 0, static_cast<size_t>(H) * K * sizeof(float), stream);
    return ce == cudaSuccess ? PT_OK : cuda_fail(ce);
  }
  DeviceInfo* di = nullptr;
  if ((rc = current_device(di)) != PT_OK) return rc;
  if (!ws || ws_bytes < pt::cl::dk_workspace_bytes(B, L, H, K, di->sm_count)) return PT_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(ws) & 15u) != 0) return PT_ERR_ALIGN;
  cudaError_t ce = pt::cl::launch_dk(dy, x, dk, B, L, H, K, accumulate ? 1 : 0, ws, di->sm_count, stream);
  return ce == cudaSuccess ? PT_OK : cuda_fail(ce);
}

int pt_config(int path, int B, int H, int L, int K, int* out, int n) {
  if (path < 0 || path > 2 || !out || n < 4) return PT_ERR_ARGS;
  if (B < 1 || H < 1 || L < 1 || K < 1) return PT_ERR_ARGS;
  if (L > PT_MAX_L || K > PT_MAX_K) return PT_ERR_UNSUPPORTED;
  std::call_once(g_once, init_once);
  const pt::LaunchCfg c = cfg_for(path, L, K);
  const pt::Entry* e = find_entry(L, K);
  out[0] = c.rows;
  out[1] = c.stages;
  out[2] = c.ctas_per_sm;
  out[3] = (e && (e->loader == pt::LOAD_TMA3D || (static_cast<long long>(H) * L) % 4 == 0)) ? 1 : 0;
  if (n >= 5) out[4] = intensity_class(L, K);
  if (n >= 6) out[5] = c.tpr;
  if (n >= 7) {
    int sm = 0, dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      sm = 0;
    (void)cudaGetLastError();
    out[6] = engine_for(path, B, H, L, K, sm);
  }
  if (n >= 9) {
    const pt::BwdChoice c = bwd_choice(L, K);
    out[7] = c.kernel;
    out[8] = c.helper_channels;
  }
  return PT_OK;
}

int pt_kernel_info(int path, int B, int H, int L, int K, int* out, int n) {
  if (path < 0 || path > PT_PATH_BWD_FUSED || !out || n < 8) return PT_ERR_ARGS;
  if (B < 1 || H < 1 || L < 1 || K < 1) return PT_ERR_ARGS;
  if (L > PT_MAX_L || K > PT_MAX_K) return PT_ERR_UNSUPPORTED;
  DeviceInfo* di = nullptr;
  int rc = current_device(di);
  if (rc != PT_OK) return rc;
  Plan p;
  if (path == PT_PATH_BWD_FUSED) {
    if (plan_backward(B, H, L, K, *di, p) == 0) return PT_ERR_UNSUPPORTED;
  } else if ((rc = plan(path, B, H, L, K, *di, p)) != PT_OK) {
    return rc;
  }
  const void* func = p.func;
  int threads = p.threads;
  size_t dyn = p.smem;
  int grid = p.g.G;
  if (!p.exact) {
    threads = (path == PT_PATH_DK) ? 128 : kGenericRows;
    dyn = 0;
    if (path == PT_PATH_FWD)
      func = conv_bucket_func<pt::OP_FWD>(L, K);
    else if (path == PT_PATH_DX)
      func = conv_bucket_func<pt::OP_DX>(L, K);
    else
      func = dk_bucket_func(L, K);
    if (path != PT_PATH_DK) {
      const long long S = static_cast<long long>(B) * H;
      const long long n_tiles = (S + kGenericRows - 1) / kGenericRows;
      long long gsz = static_cast<long long>(di->sm_count) * 8;
      grid = static_cast<int>(gsz < n_tiles ? gsz : n_tiles);
    }
  }
  cudaFuncAttributes fa;
  cudaError_t ce = cudaFuncGetAttributes(&fa, func);
  if (ce != cudaSuccess) return cuda_fail(ce);
  int occ = 0;
  ce = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, func, threads, dyn);
  if (ce != cudaSuccess) return cuda_fail(ce);
  out[0] = fa.numRegs;
  out[1] = static_cast<int>(fa.sharedSizeBytes);
  out[2] = static_cast<int>(fa.localSizeBytes);
  out[3] = threads;
  out[4] = static_cast<int>(dyn);
  out[5] = occ;
  out[6] = grid;
  out[7] = p.exact ? 1 : 0;
  return PT_OK;
}

int pt_set_config(int path, int rows_per_tile, int stages, int ctas_per_sm, int threads_per_row) {
  if (path < 0 || path > 2) return PT_ERR_ARGS;
  if (rows_per_tile == 0) {
    g_opts.has_cfg[path] = false;
    return PT_OK;
  }
  if (!cfg_valid(rows_per_tile, stages, ctas_per_sm, threads_per_row)) return PT_ERR_ARGS;
  g_opts.cfg[path] = pt::LaunchCfg{rows_per_tile, stages, ctas_per_sm, threads_per_row};
  g_opts.has_cfg[path] = true;
  return PT_OK;
}

int pt_set_engine(int path, int engine) {
  if (path < 0 || path > 2) return PT_ERR_ARGS;
  if (engine != -1 && engine != PT_ENGINE_FFMA && engine != PT_ENGINE_TENSOR) return PT_ERR_ARGS;
  g_opts.engine[path] = engine;
  return PT_OK;
}

// ---------------- per-call launch options ----------------
int pt_fwd_ex(const float* x, const float* k, float* y, int B, int H, int L, int K, const pt_launch_opts* o,
              void* stream) {
  Opts op;
  if (!to_opts(o, op)) return PT_ERR_ARGS;
  OptsScope scope(o ? &op : nullptr);
  return pt_fwd(x, k, y, B, H, L, K, stream);
}

int pt_dx_ex(const float* dy, const float* k, float* dx, int B, int H, int L, int K, const pt_launch_opts* o,
             void* stream) {
  Opts op;
  if (!to_opts(o, op)) return PT_ERR_ARGS;
  OptsScope scope(o ? &op : nullptr);
  return pt_dx(dy, k, dx, B, H, L, K, stream);
}

int pt_dk_ex(const float* dy, const float* x, float* dk, int B, int H, int L, int K, int mode, void* ws,
             size_t ws_bytes, const pt_launch_opts* o, void* stream) {
  Opts op;
  if (!to_opts(o, op)) return PT_ERR_ARGS;
  OptsScope scope(o ? &op : nullptr);
  return pt_dk(dy, x, dk, B, H, L, K, mode, ws, ws_bytes, stream);
}

int pt_dx_dk_ex(const float* dy, const float* x, const float* k, float* dx, float* dk, int B, int H, int L,
                int K, int mode, void* ws, size_t ws_bytes, const pt_launch_opts* o, void* stream) {
  Opts op;
  if (!to_opts(o, op)) return PT_ERR_ARGS;
  OptsScope scope(o ? &op : nullptr);
  return pt_dx_dk(dy, x, k, dx, dk, B, H, L, K, mode, ws, ws_bytes, stream);
}

size_t pt_dk_workspace_bytes_ex(int B, int H, int L, int K, const pt_launch_opts* o) {
  Opts op;
  if (!to_opts(o, op)) return 0;
  OptsScope scope(o ? &op : nullptr);
  return pt_dk_workspace_bytes(B, H, L, K);
}

size_t pt_dx_dk_workspace_bytes_ex(int B, int H, int L, int K, const pt_launch_opts* o) {
  Opts op;
  if (!to_opts(o, op)) return 0;
  OptsScope scope(o ? &op : nullptr);
  return pt_dx_dk_workspace_bytes(B, H, L, K);
}

int pt_dx_dk_fused_ex(int B, int H, int L, int K, const pt_launch_opts* o) {
  Opts op;
  if (!to_opts(o, op)) return 0;
  OptsScope scope(o ? &op : nullptr);
  return pt_dx_dk_fused(B, H, L, K);
}

int pt_config_ex(int path, int B, int H, int L, int K, int* out, int n, const pt_launch_opts* o) {
  Opts op;
  if (!to_opts(o, op)) return PT_ERR_ARGS;
  OptsScope scope(o ? &op : nullptr);
  return pt_config(path, B, H, L, K, out, n);
}

int pt_kernel_info_ex(int path, int B, int H, int L, int K, int* out, int n, const pt_launch_opts* o) {
  Opts op;
  if (!to_opts(o, op)) return PT_ERR_ARGS;
  OptsScope scope(o ? &op : nullptr);
  return pt_kernel_info(path, B, H, L, K, out, n);
}

// ---------------- dK summed over the ranks through peer memory ----------------
size_t pt_peer_buffer_bytes(int world, int H, int K) {
  if (world < 1 || world > PT_MAX_PEERS || H < 1 || K < 1 || K > PT_MAX_K) return 0;
  const size_t data = 2ull * world * H * K * sizeof(float);
  const size_t flags = 2ull * world * H * sizeof(unsigned);
  return (data + 255) / 256 * 256 + (flags + 255) / 256 * 256;
}

int pt_peer_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return PT_ERR_ARGS;
  *ptr = nullptr;
  DeviceInfo* di = nullptr;
  int rc = current_device(di);
  if (rc != PT_OK) return rc;
  void* p = nullptr;
  cudaError_t ce = cudaMalloc(&p, bytes);
  if (ce != cudaSuccess) return cuda_fail(ce);
  if ((ce = cudaMemset(p, 0, bytes)) != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(ce);
  }
  *ptr = p;
  return PT_OK;
}

int pt_peer_free(void* ptr) {
  if (!ptr) return PT_OK;
  const cudaError_t ce = cudaFree(ptr);
  return ce == cudaSuccess ? PT_OK : cuda_fail(ce);
}

int pt_ipc_export(const void* ptr, void* handle) {
  if (!ptr || !handle) return PT_ERR_ARGS;
  cudaIpcMemHandle_t h;
  const cudaError_t ce = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (ce != cudaSuccess) return cuda_fail(ce);
  static_assert(sizeof(h) == PT_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return PT_OK;
}

int pt_ipc_import(const void* handle, void** ptr) {
  if (!handle || !ptr) return PT_ERR_ARGS;
  *ptr = nullptr;
  DeviceInfo* di = nullptr;
  int rc = current_device(di);
  if (rc != PT_OK) return rc;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t ce = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return ce == cudaSuccess ? PT_OK : cuda_fail(ce);
}

int pt_ipc_close(void* ptr) {
  if (!ptr) return PT_OK;
  const cudaError_t ce = cudaIpcCloseMemHandle(ptr);
  return ce == cudaSuccess ? PT_OK : cuda_fail(ce);
}

namespace {

int peer_args(const pt_peer_group* grp, int H, int K, pt::PeerArgs& pa) {
  if (!grp || grp->world < 2 || grp->world > PT_MAX_PEERS || grp->rank < 0 || grp->rank >= grp->world ||
      grp->epoch == 0)
    return PT_ERR_ARGS;
  const size_t data = 2ull * grp->world * H * K * sizeof(float);
  for (int r = 0; r < grp->world; ++r) {
    if (!grp->bufs[r] || !aligned16(grp->bufs[r])) return PT_ERR_ARGS;
    pa.data[r] = static_cast<float*>(grp->bufs[r]);
    pa.flags[r] = reinterpret_cast<unsigned*>(static_cast<unsigned char*>(grp->bufs[r]) + (data + 255) / 256 * 256);
  }
  pa.rank = grp->rank;
  pa.world = grp->world;
  pa.H = H;
  pa.K = K;
  pa.epoch = grp->epoch;
  return PT_OK;
}

int launch_peer_allreduce(float* dk, const pt::PeerArgs& pa, unsigned* err, cudaStream_t stream) {
  pt::peer_allreduce_kernel<<<pa.H, 64, 0, stream>>>(dk, pa, err);
  const cudaError_t ce = cudaGetLastError();
  return ce == cudaSuccess ? PT_OK : cuda_fail(ce);
}

}  // namespace

int pt_allreduce_peer(float* dk, int H, int K, const pt_peer_group* grp, void* stream) {
  if (!dk || H < 1 || K < 1 || K > PT_MAX_K) return PT_ERR_ARGS;
  pt::PeerArgs pa{};
  int rc = peer_args(grp, H, K, pa);
  if (rc != PT_OK) return rc;
  DeviceInfo* di = nullptr;
  if ((rc = current_device(di)) != PT_OK) return rc;
  return launch_peer_allreduce(dk, pa, di->err, static_cast<cudaStream_t>(stream));
}

int pt_dx_dk_allreduce(const float* dy, const float* x, const float* k, float* dx, float* dk, int B, int H,
                       int L, int K, void* ws, size_t ws_bytes, const pt_peer_group* grp, void* stream_v) {
  int rc = check_common(dy, x, k, B, H, L, K);
  if (rc != PT_OK) return rc;
  if (!dk || (B > 0 && !dx)) return PT_ERR_ARGS;
  pt::PeerArgs pa{};
  if ((rc = peer_args(grp, H, K, pa)) != PT_OK) return rc;
  DeviceInfo* di = nullptr;
  if ((rc = current_device(di)) != PT_OK) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (B > 0) {
    Plan p;
    if (plan_backward(B, H, L, K, *di, p) == 1 && p.sched.direct)
      return launch_fused(p, dy, x, k, dx, dk, PT_DK_DETERMINISTIC, ws, di->err, stream, &pa);
  }
  if ((rc = pt_dx_dk(dy, x, k, dx, dk, B, H, L, K, PT_DK_DETERMINISTIC, ws, ws_bytes, stream_v)) != PT_OK)
    return rc;
  return launch_peer_allreduce(dk, pa, di->err, stream);
}

int pt_dx_dk_allreduce_fused(int B, int H, int L, int K) {
  if (B < 1 || H < 1 || L < 1 || K < 1 || L > PT_MAX_L || K > PT_MAX_K) return 0;
  DeviceInfo* di = nullptr;
  if (current_device(di) != PT_OK) return 0;
  Plan p;
  return (plan_backward(B, H, L, K, *di, p) == 1 && p.sched.direct) ? 1 : 0;
}

int pt_selftest_wait_timeout(unsigned long long limit_ns, void* out, void* stream) {
  if (!out || limit_ns == 0 || limit_ns > 1000000000ull) return PT_ERR_ARGS;
  if (!aligned16(out)) return PT_ERR_ALIGN;
  DeviceInfo* di = nullptr;
  int rc = current_device(di);
  if (rc != PT_OK) return rc;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      limit_ns, static_cast<unsigned long long*>(out), di->err);
  const cudaError_t ce = cudaGetLastError();
  return ce == cudaSuccess ? PT_OK : cuda_fail(ce);
}

int pt_device_error(unsigned int* out, int clear) {
  if (!out) return PT_ERR_ARGS;
  DeviceInfo* di = nullptr;
  int rc = current_device(di);
  if (rc != PT_OK) return rc;
  cudaError_t ce = cudaDeviceSynchronize();
  if (ce != cudaSuccess) return cuda_fail(ce);
  ce = cudaMemcpyFromSymbol(out, g_pt_device_error, sizeof(unsigned));
  if (ce != cudaSuccess) return cuda_fail(ce);
  if (clear) {
    const unsigned zero = 0;
    ce = cudaMemcpyToSymbol(g_pt_device_error, &zero, sizeof(unsigned));
    if (ce != cudaSuccess) return cuda_fail(ce);
  }
  return PT_OK;
}

const char* pt_status_string(int status) {
  switch (status) {
    case PT_OK: return "ok";
    case PT_ERR_ARGS: return "invalid arguments (null pointer, non-positive or mismatched dimensions)";
    case PT_ERR_UNSUPPORTED: return "unsupported shape: kernels require L <= 48 and K <= 48";
    case PT_ERR_ALIGN: return "pointer not 16-byte aligned";
    case PT_ERR_WORKSPACE: return "deterministic dK workspace missing or smaller than pt_dk_workspace_bytes()";
    case PT_ERR_CUDA: return "CUDA call or kernel launch failed (see pt_last_cuda_error)";
    case PT_ERR_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    case PT_ERR_SCRATCH_LIMIT:
      return "shape needs more dK scratch than pt_dk_noalloc's fixed 8 MiB array; use pt_dk with a workspace";
    default: return "unknown status";
  }
}

int pt_last_cuda_error(void) { return t_last_cuda_error; }

int pt_version(void) { return 100; }

}  // extern "C"
