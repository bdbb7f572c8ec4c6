// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[b] = alpha * A[b] . B[b]^T + beta * C[b]        (optional D2 = D + gamma2 * I)
//
// A is M x K and B is N x K in the MMA's view. Either operand may be stored
// K-major (rows of K contiguous) or MN-major (M/N contiguous); both are read
// with 128-byte-swizzled TMA tiles and described to the tensor core with
// matching shared-memory descriptors, so no transposed copies are ever made.
//
// Roles (320 threads):
//   warp 0      TMA producer (lane 0)
//   warp 1      TMEM allocator + MMA issuer (lane 0)
//   warps 2..9  epilogue: two warps per TMEM lane quarter (32 accumulator rows),
//               one taking the even and one the odd 32-column chunks
//
// The fp32 accumulator lives in TMEM, double buffered (2 x BN columns) so the
// epilogue of one tile overlaps the main loop of the next.
//
// Epilogue, per warp and per 32 x 32 block of its rows, in a ring of staging slots:
//   C rows   <- 16-byte loads into registers, one block ahead
//   x        = alpha * acc (tcgen05.ld) + beta * C, rounded to the output type
//   slot     <- x (row-major), TMA-stored to D / D2; in symmetric mode then
//   slot     <- x^T, TMA-stored to the mirror position (out-of-range elements clipped)
// In symmetric mode only blocks with column >= row are produced; each strictly
// upper block is also stored transposed, and the 32 x 32 diagonal blocks are
// symmetrised in shared memory and written with masked generic stores, so the
// output is exactly symmetric. Outputs whose layout a TMA store cannot express
// use the same generic path. Every wait is bounded (gns_common.cuh).
#pragma once

#include "gns_common.cuh"

namespace gns {

// Set by a GEMM CTA whose bounded wait gave up; read by gns_device_status().
__device__ int g_device_status = 0;

constexpr int kBM = 128;          // UMMA M (cta_group::1)
constexpr int kBK = 64;           // 64 x 16-bit = one 128-byte swizzle row
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter, splitting the 32-column chunks
constexpr int kGemmThreads = 32 * (2 + kEpiWarps);
constexpr int kRing = 2;      // staging slots per epilogue warp

struct GemmShape {
  int M, N, K, batch;
  int tiles_m, tiles_n;
  int tiles_per_matrix;
  int total_tiles;
  int k_blocks;
  int reverse_batch;  // 1: visit matrices last-to-first (keeps the previous launch's outputs L2-hot)
};

struct GemmEpilogue {
  void* d;
  int64_t ldd, d_bstride;
  const void* c;
  int64_t ldc, c_bstride;
  void* d2;
  int64_t ldd2, d2_bstride;
  float alpha, beta, gamma2;
  int out_bf16;     // 16-bit outputs: 1 = bf16, 0 = fp16
  int round_dtype;  // -1, or a dtype every value is rounded through before the output cast
  int has_c, has_d2;
  int tma_c, tma_d, tma_d2;  // 1 = tensor map usable, 0 = generic path
  int c_vec;                 // 1 = C rows and base 16-byte aligned (vector loads)
};

template <int BN, bool OUT_F32>
struct GemmConfig {
  static constexpr int kStages = OUT_F32 ? 3 : 4;
  static constexpr uint32_t kABytes = kBM * kBK * 2;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kRowBytes = OUT_F32 ? 128 : 64;  // one 32-element staging row
  static constexpr uint32_t kChunkBytes = 32 * kRowBytes;
  static constexpr uint32_t kEpiBytes = kEpiWarps * kRing * kChunkBytes;
  static constexpr uint32_t kTmemCols = 2 * BN;
  static constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + kEpiBytes + 512;
};

// Byte offset of (row, byte) inside a swizzled 32-row staging block. The
// pattern equals the TMA's SWIZZLE_64B (16-bit rows) / SWIZZLE_128B (fp32 rows).
template <bool OUT_F32>
__device__ __forceinline__ uint32_t stage_off(uint32_t row, uint32_t byte) {
  if (OUT_F32) return row * 128u + (byte ^ ((row & 7u) << 4));
  return row * 64u + (byte ^ (((row >> 1) & 3u) << 4));
}

// Tile index -> (matrix, row block, column block).
template <int BN, bool SYM>
__device__ __forceinline__ void decode_tile(const GemmShape& s, int t, int& b, int& i, int& j) {
  b = t / s.tiles_per_matrix;
  int l = t - b * s.tiles_per_matrix;
  if (s.reverse_batch) b = s.batch - 1 - b;
  if (!SYM) {
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

__device__ __forceinline__ uint32_t pack_half2(float a, float b, int bf16) {
  if (bf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float half_bits_to_float(uint16_t bits, int bf16) {
  if (bf16) return __bfloat162float(__ushort_as_bfloat16(bits));
  return __half2float(__ushort_as_half(bits));
}

__device__ __forceinline__ uint16_t float_to_half_bits(float v, int bf16) {
  if (bf16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  return __half_as_ushort(__float2half_rn(v));
}

// Reads row `row` (32 values) of a swizzled staging block as fp32.
template <bool OUT_F32>
__device__ __forceinline__ void stage_read_row(const uint8_t* buf, uint32_t row, int bf16, float (&x)[32]) {
  if (OUT_F32) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float4 f = *reinterpret_cast<const float4*>(buf + stage_off<true>(row, 16u * k));
      x[4 * k] = f.x; x[4 * k + 1] = f.y; x[4 * k + 2] = f.z; x[4 * k + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint4 u = *reinterpret_cast<const uint4*>(buf + stage_off<false>(row, 16u * k));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        x[8 * k + 2 * e] = half_bits_to_float(static_cast<uint16_t>(w[e] & 0xffffu), bf16);
        x[8 * k + 2 * e + 1] = half_bits_to_float(static_cast<uint16_t>(w[e] >> 16), bf16);
      }
    }
  }
}

// Writes row `row` (32 values, already rounded) of a swizzled staging block.
template <bool OUT_F32>
__device__ __forceinline__ void stage_write_row(uint8_t* buf, uint32_t row, int bf16, const float (&x)[32]) {
  if (OUT_F32) {
#pragma unroll
    for (int k = 0; k < 8; ++k)
      *reinterpret_cast<float4*>(buf + stage_off<true>(row, 16u * k)) =
          make_float4(x[4 * k], x[4 * k + 1], x[4 * k + 2], x[4 * k + 3]);
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      *reinterpret_cast<uint4*>(buf + stage_off<false>(row, 16u * k)) =
          make_uint4(pack_half2(x[8 * k], x[8 * k + 1], bf16), pack_half2(x[8 * k + 2], x[8 * k + 3], bf16),
                     pack_half2(x[8 * k + 4], x[8 * k + 5], bf16), pack_half2(x[8 * k + 6], x[8 * k + 7], bf16));
  }
}

// Writes column `col` (32 values) of a swizzled staging block: element q goes to (q, col).
template <bool OUT_F32>
__device__ __forceinline__ void stage_write_col(uint8_t* buf, uint32_t col, int bf16, const float (&x)[32]) {
#pragma unroll
  for (int q = 0; q < 32; ++q) {
    if (OUT_F32)
      *reinterpret_cast<float*>(buf + stage_off<true>(q, 4u * col)) = x[q];
    else
      *reinterpret_cast<uint16_t*>(buf + stage_off<false>(q, 2u * col)) = float_to_half_bits(x[q], bf16);
  }
}

template <bool OUT_F32>
__device__ __forceinline__ float stage_get(const uint8_t* buf, uint32_t row, uint32_t col, int bf16) {
  if (OUT_F32) return *reinterpret_cast<const float*>(buf + stage_off<true>(row, 4u * col));
  return half_bits_to_float(*reinterpret_cast<const uint16_t*>(buf + stage_off<false>(row, 2u * col)), bf16);
}

template <bool OUT_F32>
__device__ __forceinline__ void global_put(void* base, int64_t idx, float v, int bf16) {
  if (OUT_F32)
    static_cast<float*>(base)[idx] = v;
  else
    static_cast<uint16_t*>(base)[idx] = float_to_half_bits(v, bf16);
}

template <bool OUT_F32>
__device__ __forceinline__ float global_get(const void* base, int64_t idx, int bf16) {
  if (OUT_F32) return static_cast<const float*>(base)[idx];
  return half_bits_to_float(static_cast<const uint16_t*>(base)[idx], bf16);
}

// 32 consecutive accumulator-input values of one row, as raw 16-byte words.
template <bool OUT_F32>
struct CRow {
  uint4 u[OUT_F32 ? 8 : 4];
};

// Plain (coherent) 16-byte loads: C may alias D, which this kernel writes.
template <bool OUT_F32>
__device__ __forceinline__ void c_row_load(CRow<OUT_F32>& dst, const void* base, int64_t elem_off) {
  const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(base) + elem_off * (OUT_F32 ? 4 : 2));
#pragma unroll
  for (int q = 0; q < (OUT_F32 ? 8 : 4); ++q) dst.u[q] = p[q];
}

template <bool OUT_F32>
__device__ __forceinline__ void c_row_unpack(const CRow<OUT_F32>& src, int bf16, float (&x)[32]) {
#pragma unroll
  for (int q = 0; q < (OUT_F32 ? 8 : 4); ++q) {
    const uint32_t w[4] = {src.u[q].x, src.u[q].y, src.u[q].z, src.u[q].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (OUT_F32) {
        x[4 * q + e] = __uint_as_float(w[e]);
      } else {
        x[8 * q + 2 * e] = half_bits_to_float(static_cast<uint16_t>(w[e] & 0xffffu), bf16);
        x[8 * q + 2 * e + 1] = half_bits_to_float(static_cast<uint16_t>(w[e] >> 16), bf16);
      }
    }
  }
}

template <int BN, bool A_MN, bool B_MN, bool OUT_F32, bool SYM>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_c, const __grid_constant__ CUtensorMap tmap_d,
                   const __grid_constant__ CUtensorMap tmap_d2, const GemmShape shape, const GemmEpilogue epi,
                   const int ab_bf16) {
  using Cfg = GemmConfig<BN, OUT_F32>;
  constexpr int S = Cfg::kStages;
  constexpr uint32_t CB = Cfg::kChunkBytes;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + S * Cfg::kABytes;
  uint8_t* smem_epi = smem + S * Cfg::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_epi + Cfg::kEpiBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + S;
  uint64_t* tfull_bar = bars + 2 * S;
  uint64_t* tempty_bar = bars + 2 * S + 2;
  uint64_t* c_bar = bars + 2 * S + 4;  // one per ring slot of each epilogue warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(c_bar + kRing * kEpiWarps);
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
      mbar_init(&tempty_bar[a], 32 * kEpiWarps);
    }
    for (int k = 0; k < kRing * kEpiWarps; ++k) mbar_init(&c_bar[k], 1);
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
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      for (int t = blockIdx.x; t < shape.total_tiles; t += gridDim.x) {
        int b, i, j;
        decode_tile<BN, SYM>(shape, t, b, i, j);
        const int m0 = i * kBM, n0 = j * BN;
        for (int kb = 0; kb < shape.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[st], ph ^ 1u, abort_flag, &g_device_status, kStatusProducerTimeout))
            goto producer_done;
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
    // ------------------------------------------------------------ MMA issuer
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
    // ------------------------------------------------------------ epilogue
    // Each warp owns a ring of kRing staging slots. A slot holds, in turn, the
    // result block of one chunk (TMA-stored to D / D2) and, in symmetric mode,
    // its transpose (TMA-stored to the mirror position).
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const int half = ew >> 2;      // even (0) or odd (1) 32-column chunks
    uint8_t* ring = smem_epi + ew * kRing * CB;
    const int bf16 = epi.out_bf16;
    const bool use_c = epi.has_c != 0;
    constexpr int kChunks = BN / 32;
    int acc = 0;
    uint32_t acc_ph = 0;
    bool aborted = false;

    for (int t = blockIdx.x; t < shape.total_tiles && !aborted; t += gridDim.x) {
      int b, i, j;
      decode_tile<BN, SYM>(shape, t, b, i, j);
      const int r0 = i * kBM + quarter * 32;
      const int cbase = j * BN;
      // Needed chunks form the run [first, end): in range, and column >= row when symmetric.
      int end = (shape.N - cbase + 31) / 32;
      end = end < kChunks ? end : kChunks;
      int first = SYM ? ((r0 > cbase) ? (r0 - cbase) / 32 : 0) : 0;
      if (r0 >= shape.M) first = end;
      // Slots may still be read by the previous tile's stores.
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
      // C rows travel through the LSU path (not the TMA queue, where they would
      // wait behind the main loop's operand tiles), one chunk ahead in registers.
      const int64_t c_row = static_cast<int64_t>(b) * epi.c_bstride + static_cast<int64_t>(r0 + lane) * epi.ldc;
      auto c_ok = [&](int cc) { return use_c && epi.c_vec && (r0 + lane < shape.M) && (cbase + cc * 32 + 32 <= shape.N); };
      CRow<OUT_F32> c_cur, c_next;
      const int start = first + (((first & 1) != half) ? 1 : 0);  // this warp's chunks: start, start + 2, ...
      if (start < end && c_ok(start)) c_row_load<OUT_F32>(c_cur, epi.c, c_row + cbase + start * 32);
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_ph, abort_flag, &g_device_status, kStatusEpilogueTimeout)) {
        aborted = true;
        break;
      }
      __syncwarp();
      tc_fence_after();
      const uint32_t lane_addr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      int jj = 0;
#pragma unroll 1
      for (int cc = start; cc < end; cc += 2, ++jj) {
        const int c0 = cbase + cc * 32;
        const int k = jj % kRing;
        uint8_t* buf = ring + k * CB;
        if (cc + 2 < end && c_ok(cc + 2)) c_row_load<OUT_F32>(c_next, epi.c, c_row + c0 + 64);
        float v[32];
        __syncwarp();
        tmem_load_32cols(lane_addr + cc * 32, v);
        float cv[32];
        if (use_c) {
          if (c_ok(cc)) {
            c_row_unpack<OUT_F32>(c_cur, bf16, cv);
          } else {
#pragma unroll
            for (int q = 0; q < 32; ++q)
              cv[q] = (r0 + lane < shape.M && c0 + q < shape.N) ? global_get<OUT_F32>(epi.c, c_row + c0 + q, bf16) : 0.0f;
          }
          c_cur = c_next;
        }
        float x[32];
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          float y = epi.alpha * v[q];
          if (use_c) y = fmaf(epi.beta, cv[q], y);
          if (epi.round_dtype >= 0) y = round_to(y, epi.round_dtype);
          if (!OUT_F32) y = bf16 ? __bfloat162float(__float2bfloat16_rn(y)) : __half2float(__float2half_rn(y));
          x[q] = y;
        }
        const bool diag = SYM && (c0 == r0);
        const bool mirror = SYM && !diag;
        __syncwarp();  // every lane has read its C row before the slot is overwritten
        stage_write_row<OUT_F32>(buf, lane, bf16, x);
        const bool fast = !diag && epi.tma_d && (!epi.has_d2 || epi.tma_d2);
        if (fast) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmap_d, buf, c0, r0, b);
            if (epi.has_d2) tma_store_3d(&tmap_d2, buf, c0, r0, b);
            bulk_commit_group();
          }
          if (mirror) {
            if (lane == 0) bulk_wait_read_all();
            __syncwarp();
            stage_write_col<OUT_F32>(buf, lane, bf16, x);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&tmap_d, buf, r0, c0, b);
              if (epi.has_d2) tma_store_3d(&tmap_d2, buf, r0, c0, b);
              bulk_commit_group();
            }
          } else if (lane == 0) {
            bulk_wait_read_1();  // only this chunk's group may still read its slot
          }
        } else {
          // Generic path: diagonal blocks (symmetrised here) and outputs a TMA
          // store cannot express. Lane = column, loop = row: coalesced rows.
          __syncwarp();
          const int gc = c0 + lane;
          const int64_t dbb = static_cast<int64_t>(b) * epi.d_bstride;
          const int64_t d2b = static_cast<int64_t>(b) * epi.d2_bstride;
#pragma unroll 1
          for (int xr = 0; xr < 32; ++xr) {
            const int gr = r0 + xr;
            if (gr >= shape.M || gc >= shape.N) continue;
            float val;
            if (diag)
              val = (lane >= xr) ? stage_get<OUT_F32>(buf, xr, lane, bf16) : stage_get<OUT_F32>(buf, lane, xr, bf16);
            else
              val = stage_get<OUT_F32>(buf, xr, lane, bf16);
            global_put<OUT_F32>(epi.d, dbb + static_cast<int64_t>(gr) * epi.ldd + gc, val, bf16);
            if (epi.has_d2)
              global_put<OUT_F32>(epi.d2, d2b + static_cast<int64_t>(gr) * epi.ldd2 + gc,
                                  (gr == gc) ? val + epi.gamma2 : val, bf16);
          }
          if (mirror) {
            // Strictly upper block with an output a TMA store cannot express:
            // element (c0 + xr, r0 + lane) is the value computed at (r0 + lane, c0 + xr).
            const int gc2 = r0 + lane;
#pragma unroll 1
            for (int xr = 0; xr < 32; ++xr) {
              const int gr2 = c0 + xr;
              if (gr2 >= shape.M || gc2 >= shape.N) continue;
              const float val = stage_get<OUT_F32>(buf, lane, xr, bf16);
              global_put<OUT_F32>(epi.d, dbb + static_cast<int64_t>(gr2) * epi.ldd + gc2, val, bf16);
              if (epi.has_d2) global_put<OUT_F32>(epi.d2, d2b + static_cast<int64_t>(gr2) * epi.ldd2 + gc2, val, bf16);
            }
          }
          if (lane == 0) bulk_wait_read_all();
        }
        __syncwarp();
      }
      if (aborted) break;
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1u;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
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
