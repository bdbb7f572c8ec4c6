// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[b] = alpha * A[b] . B[b]^T + beta * C[b] + gamma * I
//
// A is M x K and B is N x K in the MMA's view. Either operand may be stored
// K-major (rows of K contiguous) or MN-major (M/N contiguous); both are read
// with 128-byte-swizzled TMA tiles and described to the tensor core with
// matching shared-memory descriptors, so no transposed copies are ever made.
//
// Roles (192 threads):
//   warp 0      TMA producer (lane 0)
//   warp 1      TMEM allocator + MMA issuer (lane 0)
//   warps 2..5  epilogue: TMEM -> registers -> global, one TMEM lane quarter each
//
// The fp32 accumulator lives in TMEM, double buffered (2 x BN columns) so the
// epilogue of one tile overlaps the main loop of the next. In symmetric mode
// only tiles touching the upper triangle are computed; each value with
// column >= row is written to (r, c) and mirrored to (c, r), which makes the
// output exactly symmetric. Every wait is bounded (gns_common.cuh).
#pragma once

#include "gns_common.cuh"

namespace gns {

// Set by a GEMM CTA whose bounded wait gave up; read by gns_device_status().
__device__ int g_device_status = 0;

constexpr int kBM = 128;          // UMMA M (cta_group::1)
constexpr int kBK = 64;           // 64 x 16-bit = one 128-byte swizzle row
constexpr int kGemmThreads = 192;

struct GemmShape {
  int M, N, K, batch;
  int tiles_m, tiles_n;
  int tiles_per_matrix;
  int total_tiles;
  int k_blocks;
  int symmetric;
};

struct GemmEpilogue {
  void* d;            // primary output
  int64_t ldd, d_bstride;
  int d_dtype;
  int round_dtype;    // >= 0: round to this dtype first (mirrors an intermediate cast)
  const void* c;      // optional accumulator input, read only when beta != 0
  int64_t ldc, c_bstride;
  int c_dtype;
  float alpha, beta, gamma;  // gamma is added on the diagonal
  void* d2;           // optional second output: D2 = stored(D) + gamma2 * I
  int64_t ldd2, d2_bstride;
  int d2_dtype;
  float gamma2;
  int vec_ok;         // 1 when D/C/D2 rows are 16-byte aligned for vector access
};

template <int BN>
struct GemmConfig {
  static constexpr int kStages = (BN == 256) ? 4 : 6;
  static constexpr uint32_t kABytes = kBM * kBK * 2;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kTmemCols = 2 * BN;
  static constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + 256;
};

// Tile index -> (matrix, row block, column block).
template <int BN>
__device__ __forceinline__ void decode_tile(const GemmShape& s, int t, int& b, int& i, int& j) {
  b = t / s.tiles_per_matrix;
  int l = t - b * s.tiles_per_matrix;
  if (!s.symmetric) {
    i = l / s.tiles_n;
    j = l - i * s.tiles_n;
    return;
  }
  // Row block i holds column blocks floor(128 i / BN) .. tiles_n - 1.
  for (i = 0; i < s.tiles_m; ++i) {
    const int j0 = (i * kBM) / BN;
    const int cnt = s.tiles_n - j0;
    if (l < cnt) {
      j = j0 + l;
      return;
    }
    l -= cnt;
  }
  i = s.tiles_m - 1;
  j = s.tiles_n - 1;
}

__device__ __forceinline__ uint32_t pack2(float a, float b, int dtype) {
  if (dtype == kBF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Stores 32 consecutive values of row r starting at column c0 (all in range, aligned).
__device__ __forceinline__ void store_row32(void* base, int64_t off, int dtype, const float (&x)[32]) {
  if (dtype == kF32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(base) + off);
#pragma unroll
    for (int q = 0; q < 8; ++q) p[q] = make_float4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
  } else {
    uint4* p = reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + off);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      p[q] = make_uint4(pack2(x[8 * q], x[8 * q + 1], dtype), pack2(x[8 * q + 2], x[8 * q + 3], dtype),
                        pack2(x[8 * q + 4], x[8 * q + 5], dtype), pack2(x[8 * q + 6], x[8 * q + 7], dtype));
    }
  }
}

__device__ __forceinline__ void load_row32(const void* base, int64_t off, int dtype, float (&x)[32]) {
  if (dtype == kF32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 f = p[q];
      x[4 * q] = f.x; x[4 * q + 1] = f.y; x[4 * q + 2] = f.z; x[4 * q + 3] = f.w;
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + off);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u = p[q];
      uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (dtype == kBF16) {
          __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&w[e]);
          float2 f = __bfloat1622float2(h);
          x[8 * q + 2 * e] = f.x; x[8 * q + 2 * e + 1] = f.y;
        } else {
          __half2 h = *reinterpret_cast<__half2*>(&w[e]);
          float2 f = __half22float2(h);
          x[8 * q + 2 * e] = f.x; x[8 * q + 2 * e + 1] = f.y;
        }
      }
    }
  }
}

// Epilogue for one 32-column chunk of one row held by this thread.
__device__ __forceinline__ void epilogue_chunk(const GemmEpilogue& e, const GemmShape& s, int b, int r,
                                               int c0, float (&v)[32]) {
  if (r >= s.M) return;
  const bool use_c = (e.beta != 0.0f) && (e.c != nullptr);
  const int64_t dbase = static_cast<int64_t>(b) * e.d_bstride;
  const int64_t cbase = static_cast<int64_t>(b) * e.c_bstride;
  const int64_t d2base = static_cast<int64_t>(b) * e.d2_bstride;
  const bool has_diag = (r >= c0) && (r < c0 + 32);
  const bool fast = e.vec_ok && (c0 + 32 <= s.N) && !has_diag && (!s.symmetric || c0 > r);

  if (fast) {
    float cv[32];
    if (use_c) load_row32(e.c, cbase + static_cast<int64_t>(r) * e.ldc + c0, e.c_dtype, cv);
    float x[32];
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      float t = e.alpha * v[q];
      if (use_c) t = fmaf(e.beta, cv[q], t);
      if (e.round_dtype >= 0) t = round_to(t, e.round_dtype);
      x[q] = round_to(t, e.d_dtype);
    }
    store_row32(e.d, dbase + static_cast<int64_t>(r) * e.ldd + c0, e.d_dtype, x);
    if (s.symmetric) {
#pragma unroll
      for (int q = 0; q < 32; ++q) store_from_float(e.d, dbase + static_cast<int64_t>(c0 + q) * e.ldd + r, e.d_dtype, x[q]);
    }
    if (e.d2 != nullptr) {
      // Off-diagonal chunk: D2 equals D.
      store_row32(e.d2, d2base + static_cast<int64_t>(r) * e.ldd2 + c0, e.d2_dtype, x);
      if (s.symmetric) {
#pragma unroll
        for (int q = 0; q < 32; ++q)
          store_from_float(e.d2, d2base + static_cast<int64_t>(c0 + q) * e.ldd2 + r, e.d2_dtype, x[q]);
      }
    }
    return;
  }

#pragma unroll
  for (int q = 0; q < 32; ++q) {
    const int c = c0 + q;
    if (c >= s.N || (s.symmetric && c < r)) continue;
    float t = e.alpha * v[q];
    if (use_c) t = fmaf(e.beta, load_as_float(e.c, cbase + static_cast<int64_t>(r) * e.ldc + c, e.c_dtype), t);
    if (c == r) t += e.gamma;
    if (e.round_dtype >= 0) t = round_to(t, e.round_dtype);
    const float x = round_to(t, e.d_dtype);
    store_from_float(e.d, dbase + static_cast<int64_t>(r) * e.ldd + c, e.d_dtype, x);
    if (s.symmetric && c != r) store_from_float(e.d, dbase + static_cast<int64_t>(c) * e.ldd + r, e.d_dtype, x);
    if (e.d2 != nullptr) {
      const float y = (c == r) ? x + e.gamma2 : x;
      store_from_float(e.d2, d2base + static_cast<int64_t>(r) * e.ldd2 + c, e.d2_dtype, y);
      if (s.symmetric && c != r) store_from_float(e.d2, d2base + static_cast<int64_t>(c) * e.ldd2 + r, e.d2_dtype, y);
    }
  }
}

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const GemmShape shape, const GemmEpilogue epi, const int ab_bf16) {
  using Cfg = GemmConfig<BN>;
  constexpr int S = Cfg::kStages;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + S * Cfg::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + S;
  uint64_t* tfull_bar = bars + 2 * S;
  uint64_t* tempty_bar = bars + 2 * S + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int st = 0; st < S; ++st) {
      mbar_init(&full_bar[st], 1);
      mbar_init(&empty_bar[st], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      for (int t = blockIdx.x; t < shape.total_tiles; t += gridDim.x) {
        int b, i, j;
        decode_tile<BN>(shape, t, b, i, j);
        const int m0 = i * kBM, n0 = j * BN;
        for (int kb = 0; kb < shape.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[st], ph ^ 1u, abort_flag, &g_device_status, kStatusProducerTimeout)) goto producer_done;
          mbar_arrive_expect_tx(&full_bar[st], Cfg::kStageBytes);
          const int k0 = kb * kBK;
          uint8_t* sa = smem_a + st * Cfg::kABytes;
          uint8_t* sb = smem_b + st * Cfg::kBBytes;
          if (!A_MN) {
            tma_load_3d(sa, &tmap_a, &full_bar[st], k0, m0, b);
          } else {
#pragma unroll
            for (int ch = 0; ch < kBM / 64; ++ch) tma_load_3d(sa + ch * 8192, &tmap_a, &full_bar[st], m0 + 64 * ch, k0, b);
          }
          if (!B_MN) {
            tma_load_3d(sb, &tmap_b, &full_bar[st], k0, n0, b);
          } else {
#pragma unroll
            for (int ch = 0; ch < BN / 64; ++ch) tma_load_3d(sb + ch * 8192, &tmap_b, &full_bar[st], n0 + 64 * ch, k0, b);
          }
          if (++st == S) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(ab_bf16, A_MN ? 1 : 0, B_MN ? 1 : 0, kBM, BN);
      int st = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      for (int t = blockIdx.x; t < shape.total_tiles; t += gridDim.x) {
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_ph ^ 1u, abort_flag, &g_device_status, kStatusMmaTimeout)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < shape.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&full_bar[st], ph, abort_flag, &g_device_status, kStatusMmaTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem_a + st * Cfg::kABytes);
          const uint32_t b_base = smem_u32(smem_b + st * Cfg::kBBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // K-major: advance 16 elements (32 bytes) inside the swizzle row.
            // MN-major: advance 16 K-rows (2 x 1024-byte swizzle atoms); LBO = 8 KB chunk stride.
            const uint64_t adesc = A_MN ? make_smem_desc_sw128(a_base + kk * 2048, 8192, 1024)
                                        : make_smem_desc_sw128(a_base + kk * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? make_smem_desc_sw128(b_base + kk * 2048, 8192, 1024)
                                        : make_smem_desc_sw128(b_base + kk * 32, 16, 1024);
            tc_mma_f16(d_tmem, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty_bar[st]);
          if (++st == S) {
            st = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tfull_bar[acc]);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1u;
      }
    }
  } else {
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int t = blockIdx.x; t < shape.total_tiles; t += gridDim.x) {
      int b, i, j;
      decode_tile<BN>(shape, t, b, i, j);
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_ph, abort_flag, &g_device_status, kStatusEpilogueTimeout)) break;
      __syncwarp();
      tc_fence_after();
      const int r = i * kBM + quarter * 32 + lane;
      const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        float v[32];
        __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the divergent stores
        tmem_load_32cols(lane_addr + cc * 32, v);
        epilogue_chunk(epi, shape, b, r, j * BN + cc * 32, v);
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1u;
    }
  }

  // Teardown: all roles meet; on abort give in-flight TMA/MMA work time to land
  // before TMEM and shared memory are released.
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) settle_for_ns(2000000ull);
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace gns
