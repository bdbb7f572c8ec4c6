// Host launch path of the tcgen05 GEMM: layout detection, TMA descriptor
// encoding and instantiation dispatch, plus library-wide error plumbing.
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/gns_b200.h"
#include "gemm_sm100.cuh"
#include "gns_host.h"

namespace gns {

namespace {
thread_local std::string t_last_error;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

// Optional per-launch GEMM timing (gns_profile_enable / gns_profile_collect):
// a CUDA event pair around every GEMM launch, plus its algorithmic flop count.
// The event pairs are created up front so that a launch only records them.
struct ProfileRecord {
  cudaEvent_t start, stop;
  double flops;
  int symmetric;
};
std::mutex g_prof_mutex;
bool g_prof_on = false;
int g_prof_used = 0;
std::vector<ProfileRecord> g_prof;

void profile_release() {
  for (auto& r : g_prof) {
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  g_prof.clear();
  g_prof_used = 0;
  g_prof_on = false;
}

constexpr int kMaxDevices = 64;
std::mutex g_dev_mutex;
int g_sm_count[kMaxDevices] = {0};
std::atomic<int> g_gemm_sm_limit{0};
int g_cc_major[kMaxDevices] = {0};
uint64_t g_attr_done[kMaxDevices] = {0};
int g_max_pairs[kMaxDevices][64] = {};  // co-resident CTA pairs per pair-mode instantiation
}  // namespace

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(GNS_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

void clear_error() { t_last_error.clear(); }

const char* last_error_cstr() { return t_last_error.c_str(); }

static int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(GNS_ERR_DEVICE, "device index out of range");
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  if (g_sm_count[*dev] == 0) {
    int sms = 0, major = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, *dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, *dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(cc major)");
    g_cc_major[*dev] = major;
    g_sm_count[*dev] = sms;
  }
  return GNS_OK;
}

int device_sm_count() {
  int dev = 0;
  if (current_device(&dev) != GNS_OK) return 148;
  return g_sm_count[dev];
}

int check_device() {
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != GNS_OK) return rc;
  if (g_cc_major[dev] != 10) return fail(GNS_ERR_DEVICE, "gns_b200 kernels need an sm_100 (B200) device");
  return GNS_OK;
}

namespace {

CUtensorMapDataType tma_dtype(int dtype) {
  return dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// Encodes a 3-D tensor map [batch][outer][inner] with a {64, box_outer, 1} box and 128-byte swizzle.
int make_map(CUtensorMap* map, int dtype, const void* ptr, int64_t inner, int64_t outer, int64_t batch,
             int64_t outer_stride, int64_t batch_stride, int box_outer) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return fail(GNS_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const int64_t es = 2;
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
    return fail(GNS_ERR_LAYOUT, "operand base address must be 16-byte aligned");
  if (outer == 1) outer_stride = round_up(inner, 8);
  if (batch == 1) batch_stride = round_up(outer_stride * outer, 8);
  if ((outer_stride * es) % 16 != 0 || (batch_stride * es) % 16 != 0)
    return fail(GNS_ERR_LAYOUT, "operand strides must be multiples of 16 bytes");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(outer_stride * es), static_cast<cuuint64_t>(batch_stride * es)};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_outer), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(map, tma_dtype(dtype), 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GNS_ERR_LAYOUT, "cuTensorMapEncodeTiled rejected operand layout");
  return GNS_OK;
}

// Decides whether a logical [rows, k] operand (A-style: rows = M) is K-major.
// Returns 0 = K-major, 1 = MN-major, -1 = unsupported.
int operand_major(int64_t rows, int64_t k, int64_t rstride, int64_t cstride) {
  const bool k_unit = (cstride == 1) || (k == 1);
  const bool mn_unit = (rstride == 1) || (rows == 1);
  if (k_unit && ((rstride * 2) % 16 == 0 || rows == 1)) return 0;
  if (mn_unit && ((cstride * 2) % 16 == 0 || k == 1)) return 1;
  return -1;
}

template <int BN, bool AMN, bool BMN, bool F32, bool SYM, bool PAIR, bool UP>
int launch_instance(const CUtensorMap* maps, const GemmShape& shape, const GemmEpilogue& epi, int ab_bf16,
                    cudaStream_t stream, int dev, int slot) {
  auto kern = gemm_tc_kernel<BN, AMN, BMN, F32, SYM, PAIR, UP>;
  const size_t smem = GemmConfig<BN, F32, PAIR>::kSmemBytes;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2];
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  // Programmatic dependent launch: the kernel's set-up may overlap the tail of
  // the previous kernel in the stream (it waits for it before reading data).
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (PAIR) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  int max_pairs = 0;
  {
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (!(g_attr_done[dev] & (1ull << slot))) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(smem)");
      if (PAIR) {
        // Persistent grid: as many pairs as can be resident at once.
        cfg.gridDim = dim3(2 * (g_sm_count[dev] / 2), 1, 1);
        int n = 0;
        e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
        if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
        if (n < 1) return fail(GNS_ERR_UNSUPPORTED, "no CTA pair of the GEMM fits on an SM pair");
        g_max_pairs[dev][slot] = n;
      }
      g_attr_done[dev] |= (1ull << slot);
    }
    max_pairs = g_max_pairs[dev][slot];
  }
  // Optional cap on the SMs a launch occupies (gns_set_gemm_sm_limit), so that
  // kernels running beside it (collectives) keep their SMs and no CTA of the
  // persistent grid waits for one.
  const int limit = g_gemm_sm_limit.load();
  int grid;
  if (PAIR) {
    if (limit >= 2 && limit / 2 < max_pairs) max_pairs = limit / 2;
    grid = 2 * (shape.total_tiles < max_pairs ? shape.total_tiles : max_pairs);
  } else {
    const int sms = (limit >= 1 && limit < g_sm_count[dev]) ? limit : g_sm_count[dev];
    grid = shape.total_tiles < sms ? shape.total_tiles : sms;
  }
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  ProfileRecord* rec = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_prof_mutex);
    if (g_prof_on && g_prof_used < static_cast<int>(g_prof.size())) rec = &g_prof[g_prof_used++];
  }
  if (rec) {
    // Algorithmic flops: symmetric products count the computed triangle only.
    const double mnk = static_cast<double>(shape.M) * shape.N * shape.K * shape.batch;
    rec->flops = SYM ? mnk : 2.0 * mnk;
    rec->symmetric = SYM ? 1 : 0;
    cudaEventRecord(rec->start, stream);
  }
  cudaError_t le = cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], maps[3], shape, epi, ab_bf16);
  if (le != cudaSuccess) return cuda_fail(le, "gemm kernel launch");
  if (rec) cudaEventRecord(rec->stop, stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm kernel launch");
  return GNS_OK;
}

template <int BN, bool F32, bool SYM, bool PAIR>
int dispatch_majors(int a_major, int b_major, const CUtensorMap* maps, const GemmShape& s, const GemmEpilogue& epi,
                    int bf16, cudaStream_t stream, int dev) {
  const int base = (PAIR ? 16 : 0) + (F32 ? 8 : 0) + (SYM ? 4 : 0);
  if (a_major == 0 && b_major == 0)
    return launch_instance<BN, false, false, F32, SYM, PAIR, false>(maps, s, epi, bf16, stream, dev, base + 0);
  if (a_major == 0 && b_major == 1)
    return launch_instance<BN, false, true, F32, SYM, PAIR, false>(maps, s, epi, bf16, stream, dev, base + 1);
  if (a_major == 1 && b_major == 0)
    return launch_instance<BN, true, false, F32, SYM, PAIR, false>(maps, s, epi, bf16, stream, dev, base + 2);
  return launch_instance<BN, true, true, F32, SYM, PAIR, false>(maps, s, epi, bf16, stream, dev, base + 3);
}

// Instantiations with upper-stored operands: the chains' layouts only (K-major
// A and B for symmetric products with 16-bit outputs; Q X and X Q products).
template <int BN, bool PAIR>
int dispatch_upper(bool f32, bool sym, int a_major, int b_major, const CUtensorMap* maps, const GemmShape& s,
                   const GemmEpilogue& epi, int bf16, cudaStream_t stream, int dev) {
  const int base = 32 + (PAIR ? 16 : 0) + (f32 ? 8 : 0) + (sym ? 4 : 0);
  if (sym && !f32 && a_major == 0 && b_major == 0)
    return launch_instance<BN, false, false, false, true, PAIR, true>(maps, s, epi, bf16, stream, dev, base + 0);
  if (!sym && a_major == 0 && b_major == 0) {
    if (f32) return launch_instance<BN, false, false, true, false, PAIR, true>(maps, s, epi, bf16, stream, dev, base);
    return launch_instance<BN, false, false, false, false, PAIR, true>(maps, s, epi, bf16, stream, dev, base);
  }
  if (!sym && a_major == 0 && b_major == 1) {
    if (f32)
      return launch_instance<BN, false, true, true, false, PAIR, true>(maps, s, epi, bf16, stream, dev, base + 1);
    return launch_instance<BN, false, true, false, false, PAIR, true>(maps, s, epi, bf16, stream, dev, base + 1);
  }
  return fail(GNS_ERR_UNSUPPORTED, "no instantiation for this layout with upper-stored operands");
}

template <int BN, bool PAIR>
int dispatch_outputs(bool f32, bool sym, int a_major, int b_major, const CUtensorMap* maps, const GemmShape& s,
                     const GemmEpilogue& epi, int bf16, cudaStream_t stream, int dev) {
  if (s.a_upper || s.b_upper) return dispatch_upper<BN, PAIR>(f32, sym, a_major, b_major, maps, s, epi, bf16, stream, dev);
  if (f32) {
    if (sym) return dispatch_majors<BN, true, true, PAIR>(a_major, b_major, maps, s, epi, bf16, stream, dev);
    return dispatch_majors<BN, true, false, PAIR>(a_major, b_major, maps, s, epi, bf16, stream, dev);
  }
  if (sym) return dispatch_majors<BN, false, true, PAIR>(a_major, b_major, maps, s, epi, bf16, stream, dev);
  return dispatch_majors<BN, false, false, PAIR>(a_major, b_major, maps, s, epi, bf16, stream, dev);
}

}  // namespace

int launch_gemm(const GemmArgs& g, cudaStream_t stream) {
  if (g.ab_dtype != kF16 && g.ab_dtype != kBF16) return fail(GNS_ERR_ARGUMENT, "A/B dtype must be F16 or BF16");
  if (g.batch < 0 || g.m < 0 || g.n < 0 || g.k < 0) return fail(GNS_ERR_ARGUMENT, "negative dimension");
  if (g.symmetric && g.m != g.n) return fail(GNS_ERR_ARGUMENT, "symmetric product needs m == n");
  if (g.m > (1 << 24) || g.n > (1 << 24) || g.k > (1 << 30) || g.batch > (1 << 24))
    return fail(GNS_ERR_UNSUPPORTED, "dimension beyond kernel limits");
  if (g.d_dtype < 0 || g.d_dtype > 2) return fail(GNS_ERR_ARGUMENT, "bad output dtype");
  const bool has_c = (g.c != nullptr) && (g.beta != 0.0f);
  if (has_c && g.c_dtype != g.d_dtype) return fail(GNS_ERR_ARGUMENT, "accumulator and output dtypes must match");
  if (g.d2 != nullptr && (!g.symmetric || g.d2_dtype != g.d_dtype))
    return fail(GNS_ERR_ARGUMENT, "a second output needs a symmetric product of the same dtype");
  if (g.batch == 0 || g.m == 0 || g.n == 0) return GNS_OK;
  if (g.d == nullptr) return fail(GNS_ERR_ARGUMENT, "null output");
  if (g.k == 0) return fail(GNS_ERR_UNSUPPORTED, "k == 0 products are not supported");
  int rc = check_device();
  if (rc != GNS_OK) return rc;
  int dev = 0;
  cudaGetDevice(&dev);

  // A: logical [m, k]; B: logical [k, n], as an MMA operand [n, k] with strides (cstride, rstride).
  const int a_major = operand_major(g.m, g.k, g.a.rstride, g.a.cstride);
  const int b_major = operand_major(g.n, g.k, g.b.cstride, g.b.rstride);
  if (a_major < 0 || b_major < 0) return fail(GNS_ERR_LAYOUT, "A/B need a unit stride along rows or columns");

  constexpr int BN = 256;
  // CTA pairs (256-row tiles) whenever a matrix has more than one 128-row block.
  const bool pair = g.m > kBM;
  const int tile_m = pair ? 2 * kBM : kBM;
  CUtensorMap maps[4];  // A, B, and the transposed-tile maps of upper-stored operands
  if (a_major == 0)
    rc = make_map(&maps[0], g.ab_dtype, g.a.ptr, g.k, g.m, g.batch, g.a.rstride, g.a.bstride, kBM);
  else
    rc = make_map(&maps[0], g.ab_dtype, g.a.ptr, g.m, g.k, g.batch, g.a.cstride, g.a.bstride, 64);
  if (rc != GNS_OK) return rc;
  if (b_major == 0)
    rc = make_map(&maps[1], g.ab_dtype, g.b.ptr, g.k, g.n, g.batch, g.b.cstride, g.b.bstride, pair ? BN / 2 : BN);
  else
    rc = make_map(&maps[1], g.ab_dtype, g.b.ptr, g.n, g.k, g.batch, g.b.rstride, g.b.bstride, 64);
  if (rc != GNS_OK) return rc;
  // An upper-stored symmetric operand is square and K-major; its tiles below the
  // block diagonal are read transposed through a second map of the same memory
  // with 64 x 64 boxes (the MN-major operand boxes).
  if ((g.a_upper && (a_major != 0 || g.m != g.k)) || (g.b_upper && (b_major != 0 || g.n != g.k)))
    return fail(GNS_ERR_LAYOUT, "an upper-stored operand must be square and K-major");
  if (g.upper_out && !g.symmetric)
    return fail(GNS_ERR_ARGUMENT, "upper block storage of the output needs a symmetric product");
  maps[2] = maps[0];
  maps[3] = maps[1];
  if (g.a_upper) {
    rc = make_map(&maps[2], g.ab_dtype, g.a.ptr, g.k, g.m, g.batch, g.a.rstride, g.a.bstride, 64);
    if (rc != GNS_OK) return rc;
  }
  if (g.b_upper) {
    rc = make_map(&maps[3], g.ab_dtype, g.b.ptr, g.k, g.n, g.batch, g.b.cstride, g.b.bstride, 64);
    if (rc != GNS_OK) return rc;
  }

  GemmEpilogue epi{};
  epi.d = g.d;
  epi.ldd = g.d_rstride;
  epi.d_bstride = g.d_bstride;
  epi.c = has_c ? g.c : nullptr;
  epi.ldc = g.c_rstride;
  epi.c_bstride = g.c_bstride;
  epi.d2 = g.d2;
  epi.ldd2 = g.d2_rstride;
  epi.d2_bstride = g.d2_bstride;
  epi.alpha = g.alpha;
  epi.beta = has_c ? g.beta : 0.0f;
  epi.gamma2 = g.gamma2;
  epi.out_bf16 = g.d_dtype == kBF16 ? 1 : 0;
  epi.round_dtype = g.round_dtype;
  epi.has_c = has_c ? 1 : 0;
  epi.has_d2 = g.d2 != nullptr ? 1 : 0;
  epi.upper_out = g.upper_out ? 1 : 0;
  {
    // 16-byte vector access needs an aligned base and row / batch strides.
    const int64_t es = dtype_size(g.d_dtype);
    auto aligned = [&](const void* p, int64_t rstride, int64_t bstride) {
      return reinterpret_cast<uintptr_t>(p) % 16 == 0 && (rstride * es) % 16 == 0 &&
             (g.batch == 1 || (bstride * es) % 16 == 0);
    };
    epi.c_vec = has_c && aligned(g.c, g.c_rstride, g.c_bstride) ? 1 : 0;
    epi.vec_d = aligned(g.d, g.d_rstride, g.d_bstride) ? 1 : 0;
    epi.vec_d2 = g.d2 != nullptr && aligned(g.d2, g.d2_rstride, g.d2_bstride) ? 1 : 0;
  }

  GemmShape s{};
  s.M = static_cast<int>(g.m);
  s.N = static_cast<int>(g.n);
  s.K = static_cast<int>(g.k);
  s.batch = static_cast<int>(g.batch);
  s.tiles_m = static_cast<int>((g.m + tile_m - 1) / tile_m);
  s.tiles_n = static_cast<int>((g.n + BN - 1) / BN);
  if (g.symmetric) {
    int cnt = 0;
    for (int i = 0; i < s.tiles_m; ++i) cnt += s.tiles_n - (i * tile_m) / BN;
    s.tiles_per_matrix = cnt;
  } else {
    s.tiles_per_matrix = s.tiles_m * s.tiles_n;
  }
  const int64_t total = static_cast<int64_t>(s.tiles_per_matrix) * g.batch;
  if (total > (1ll << 31) - 1) return fail(GNS_ERR_UNSUPPORTED, "too many tiles");
  s.total_tiles = static_cast<int>(total);
  s.k_blocks = static_cast<int>((g.k + kBK - 1) / kBK);
  s.reverse_batch = g.reverse_batch ? 1 : 0;
  s.a_upper = g.a_upper ? 1 : 0;
  s.b_upper = g.b_upper ? 1 : 0;

  const int bf16 = g.ab_dtype == kBF16 ? 1 : 0;
  const bool f32 = g.d_dtype == kF32;
  if (pair) return dispatch_outputs<BN, true>(f32, g.symmetric, a_major, b_major, maps, s, epi, bf16, stream, dev);
  return dispatch_outputs<BN, false>(f32, g.symmetric, a_major, b_major, maps, s, epi, bf16, stream, dev);
}

}  // namespace gns

namespace gns {
int encode_f16_tiles(CUtensorMap* map, const void* ptr, int64_t inner, int64_t outer, int64_t batch,
                     int64_t outer_stride, int64_t batch_stride, int box_outer) {
  return make_map(map, kF16, ptr, inner, outer, batch, outer_stride, batch_stride, box_outer);
}
}  // namespace gns

extern "C" {

int gns_version(void) { return 100; }

const char* gns_last_error(void) { return gns::last_error_cstr(); }

int gns_profile_enable(int capacity) {
  gns::clear_error();
  if (capacity < 0) return gns::fail(GNS_ERR_ARGUMENT, "negative profile capacity");
  std::lock_guard<std::mutex> lock(gns::g_prof_mutex);
  gns::profile_release();
  gns::g_prof.resize(static_cast<size_t>(capacity));
  for (auto& r : gns::g_prof) {
    cudaError_t e = cudaEventCreate(&r.start);
    if (e == cudaSuccess) e = cudaEventCreate(&r.stop);
    if (e != cudaSuccess) {
      gns::g_prof.resize(static_cast<size_t>(&r - gns::g_prof.data()));
      gns::profile_release();
      return gns::cuda_fail(e, "profile events");
    }
  }
  gns::g_prof_on = capacity > 0;
  return GNS_OK;
}

int gns_profile_collect(int capacity, int* count, float* ms, double* flops, int* symmetric) {
  gns::clear_error();
  if (count == nullptr) return gns::fail(GNS_ERR_ARGUMENT, "null count");
  std::lock_guard<std::mutex> lock(gns::g_prof_mutex);
  int n = 0;
  int rc = GNS_OK;
  for (int i = 0; i < gns::g_prof_used && n < capacity; ++i, ++n) {
    const auto& r = gns::g_prof[static_cast<size_t>(i)];
    float t = 0.0f;
    cudaError_t e = cudaEventSynchronize(r.stop);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&t, r.start, r.stop);
    if (e != cudaSuccess && rc == GNS_OK) rc = gns::cuda_fail(e, "profile event");
    if (ms) ms[n] = t;
    if (flops) flops[n] = r.flops;
    if (symmetric) symmetric[n] = r.symmetric;
  }
  *count = n;
  gns::profile_release();
  return rc;
}

int gns_set_gemm_sm_limit(int sms) {
  if (sms < 0) sms = 0;
  return gns::g_gemm_sm_limit.exchange(sms);
}

int gns_device_status(int* status, int clear) {
  if (status == nullptr) return gns::fail(GNS_ERR_ARGUMENT, "null status pointer");
  cudaError_t e = cudaMemcpyFromSymbol(status, gns::g_device_status, sizeof(int));
  if (e != cudaSuccess) return gns::cuda_fail(e, "read device status");
  if (clear) {
    int zero = 0;
    e = cudaMemcpyToSymbol(gns::g_device_status, &zero, sizeof(int));
    if (e != cudaSuccess) return gns::cuda_fail(e, "clear device status");
  }
  int norm = 0;
  int rc = gns::normalize_status(&norm, clear);
  if (rc != GNS_OK) return rc;
  if (*status == 0) *status = norm;
  int small = 0;
  rc = gns::small_chain_status(&small, clear);
  if (rc != GNS_OK) return rc;
  if (*status == 0) *status = small;
  return GNS_OK;
}

int gns_gemm(int ab_dtype, int64_t batch, int64_t m, int64_t n, int64_t k, const void* a, int64_t a_bstride,
             int64_t a_rstride, int64_t a_cstride, const void* b, int64_t b_bstride, int64_t b_rstride,
             int64_t b_cstride, const void* c, int c_dtype, int64_t c_bstride, int64_t c_rstride, void* d, int d_dtype,
             int64_t d_bstride, int64_t d_rstride, float alpha, float beta, int symmetric, gns_stream_t stream) {
  gns::clear_error();
  gns::GemmArgs g{};
  g.ab_dtype = ab_dtype;
  g.batch = batch;
  g.m = m;
  g.n = n;
  g.k = k;
  g.a = {a, a_bstride, a_rstride, a_cstride};
  g.b = {b, b_bstride, b_rstride, b_cstride};
  g.c = (beta != 0.0f) ? c : nullptr;
  g.c_dtype = c_dtype;
  g.c_bstride = c_bstride;
  g.c_rstride = c_rstride;
  g.d = d;
  g.d_dtype = d_dtype;
  g.d_bstride = d_bstride;
  g.d_rstride = d_rstride;
  g.round_dtype = -1;
  g.d2 = nullptr;
  g.alpha = alpha;
  g.beta = beta;
  g.symmetric = symmetric;
  if (beta != 0.0f && c == nullptr) return gns::fail(GNS_ERR_ARGUMENT, "beta != 0 needs an accumulator");
  if (c != nullptr && beta != 0.0f && (c_dtype < 0 || c_dtype > 2)) return gns::fail(GNS_ERR_ARGUMENT, "bad C dtype");
  return gns::launch_gemm(g, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
