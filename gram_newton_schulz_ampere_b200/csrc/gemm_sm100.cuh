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
// Epilogue, per warp and per 32 x 32 block of its rows (lane = row):
//   C rows   <- 16-byte loads into registers, two blocks ahead
//   x        = alpha * acc (tcgen05.ld) + beta * C, rounded to the output type
//   slot 0   <- x (row-major); in symmetric mode slot 1 <- x^T
//   D / D2   <- the slots re-read by rows, 16-byte coalesced stores
// Plain stores leave the warp at once, so no block waits for an earlier one's
// stores (a TMA store's shared-memory read completes only microseconds later,
// which made the stores the epilogue's bottleneck).
// In symmetric mode only blocks with column >= row are produced; each strictly
// upper block is also stored transposed, and the 32 x 32 diagonal blocks are
// symmetrised from the two slots, so the output is exactly symmetric. Blocks on
// the matrix edge and outputs with unaligned rows take a per-element path.
// Every wait is bounded (gns_common.cuh).
#pragma once

#include "gns_common.cuh"

namespace gns {

// Set by a GEMM CTA whose bounded wait gave up; read by gns_device_status().
__device__ int g_device_status = 0;

constexpr int kBM = 128;          // UMMA M (cta_group::1)
constexpr int kBK = 64;           // 64 x 16-bit = one 128-byte swizzle row
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter, splitting the 32-column chunks
constexpr int kGemmThreads = 32 * (2 + kEpiWarps);
constexpr int kRing = 2;      // staging slots per epilogue warp (a block and its transpose)

struct GemmShape {
  int M, N, K, batch;
  int tiles_m, tiles_n;
  int tiles_per_matrix;
  int total_tiles;
  int k_blocks;
  int reverse_batch;  // 1: visit matrices last-to-first (keeps the previous launch's outputs L2-hot)
  // 1: the K-major operand is a symmetric matrix stored as its upper block
  // triangle (256 x 256 blocks with column block >= row block); a k-block whose
  // tile lies below the block diagonal is loaded transposed (MN-major) from the
  // mirror-image tile, which is stored.
  int a_upper, b_upper;
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
  int vec_d, vec_d2;         // 1 = base, row and batch strides 16-byte aligned (vector stores)
  int upper_out;             // symmetric mode: store computed tiles as they are (upper block triangle), no mirror
  int c_vec;                 // 1 = C rows and base 16-byte aligned (vector loads)
};

// PAIR: a cluster of two CTAs computes a (2 kBM) x BN tile with cta_group::2
// MMAs; each CTA loads its 128 rows of A and half of the tile's B rows, so a
// stage is 32 KB instead of 48 KB and six fit in shared memory.
template <int BN, bool OUT_F32, bool PAIR>
struct GemmConfig {
  static constexpr int kStages = PAIR ? 5 : (OUT_F32 ? 3 : 4);
  static constexpr int kTileM = PAIR ? 2 * kBM : kBM;  // rows of one tile
  static constexpr int kBRows = PAIR ? BN / 2 : BN;    // rows of B this CTA loads
  static constexpr uint32_t kABytes = kBM * kBK * 2;
  static constexpr uint32_t kBBytes = kBRows * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kRowBytes = OUT_F32 ? 128 : 64;  // one 32-element staging row
  static constexpr uint32_t kChunkBytes = 32 * kRowBytes;
  static constexpr uint32_t kEpiBytes = kEpiWarps * kRing * kChunkBytes;
  // Pair mode, 16-bit C: each epilogue warp streams its C blocks into a ring of
  // two 32 x 32 slots with cp.async (the other modes prefetch C into registers).
  static constexpr bool kCRing = PAIR && !OUT_F32;
  static constexpr uint32_t kCRingBytes = kCRing ? kEpiWarps * 2 * kChunkBytes : 0;
  static constexpr uint32_t kTmemCols = 2 * BN;
  static constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + kEpiBytes + kCRingBytes + 512;
};

// Byte offset of (row, byte) inside a swizzled 32-row staging block. The
// pattern equals the TMA's SWIZZLE_64B (16-bit rows) / SWIZZLE_128B (fp32 rows).
template <bool OUT_F32>
__device__ __forceinline__ uint32_t stage_off(uint32_t row, uint32_t byte) {
  if (OUT_F32) return row * 128u + (byte ^ ((row & 7u) << 4));
  return row * 64u + (byte ^ (((row >> 1) & 3u) << 4));
}

// Tile index -> (matrix, row block, column block); row blocks are TILE_M rows.
template <int BN, bool SYM, int TILE_M>
__device__ __forceinline__ void decode_tile(const GemmShape& s, int t, int& b, int& i, int& j) {
  b = t / s.tiles_per_matrix;
  int l = t - b * s.tiles_per_matrix;
  if (s.reverse_batch) b = s.batch - 1 - b;
  if constexpr (!SYM) {
    i = l / s.tiles_n;
    j = l - i * s.tiles_n;
  } else {
    // Row block i holds column blocks floor(TILE_M i / BN) .. tiles_n - 1.
    for (i = 0; i < s.tiles_m; ++i) {
      const int j0 = (i * TILE_M) / BN;
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
}

// Two values rounded to 16 bits (round to nearest even), the first in the low half.
__device__ __forceinline__ uint32_t pack_pair(float a, float b, int bf16) {
  if (bf16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float half_bits_to_float(uint16_t bits, int bf16) {
  if (bf16) return __bfloat162float(__ushort_as_bfloat16(bits));
  return __half2float(__ushort_as_half(bits));
}

__device__ __forceinline__ uint16_t float_to_half_bits(float v, int bf16) {
  if (bf16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  return __half_as_ushort(__float2half_rn(v));
}

// One lane's 32 results of a chunk, already rounded to the output type: fp32
// bit patterns, or 16-bit values packed in pairs (element 2i in the low half).
template <bool OUT_F32>
struct XRow {
  uint32_t w[OUT_F32 ? 32 : 16];
};

// Writes row `row` of a swizzled staging block.
template <bool OUT_F32>
__device__ __forceinline__ void stage_write_row(uint8_t* buf, uint32_t row, const XRow<OUT_F32>& x) {
  constexpr int kVec = OUT_F32 ? 8 : 4;
#pragma unroll
  for (int k = 0; k < kVec; ++k)
    *reinterpret_cast<uint4*>(buf + stage_off<OUT_F32>(row, 16u * k)) =
        make_uint4(x.w[4 * k], x.w[4 * k + 1], x.w[4 * k + 2], x.w[4 * k + 3]);
}

// Writes column `col` (= the lane) of a swizzled staging block: element q goes
// to (q, col). 16-bit values go as 32-bit words of two adjacent columns built
// from lane pairs: per pair of rows (q, q + 1) the even lane stores row q and
// the odd lane row q + 1, each with one value received from its partner.
template <bool OUT_F32>
__device__ __forceinline__ void stage_write_col(uint8_t* buf, uint32_t col, const XRow<OUT_F32>& x) {
  if (OUT_F32) {
#pragma unroll
    for (int q = 0; q < 32; ++q) *reinterpret_cast<uint32_t*>(buf + stage_off<true>(q, 4u * col)) = x.w[q];
  } else {
    const bool odd = (col & 1u) != 0;
    const uint32_t even_col = col & ~1u;
#pragma unroll
    for (int q = 0; q < 32; q += 2) {
      const uint32_t lo = x.w[q >> 1] & 0xffffu, hi = x.w[q >> 1] >> 16;  // elements q, q + 1
      const uint32_t got = __shfl_xor_sync(0xffffffffu, odd ? lo : hi, 1);
      const uint32_t row = odd ? static_cast<uint32_t>(q + 1) : static_cast<uint32_t>(q);
      const uint32_t word = odd ? (got | (hi << 16)) : (lo | (got << 16));
      *reinterpret_cast<uint32_t*>(buf + stage_off<false>(row, 2u * even_col)) = word;
    }
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

// The C block of rows [r0, r0 + 32) and 32 columns, loaded coalesced: for each
// pass, lane L reads 16 bytes of row pass * kRows + L / kPieces (8 rows of 64
// bytes per instruction for 16-bit C, 4 rows of 128 bytes for fp32). Rows at
// or past `rows_valid` read as zero. Plain (coherent) loads: C may alias D.
template <bool OUT_F32>
__device__ __forceinline__ void c_block_load(CRow<OUT_F32>& dst, const void* base, int64_t elem_off, int64_t ldc,
                                             int rows_valid, int lane) {
  constexpr int kPieces = OUT_F32 ? 8 : 4;
  constexpr int kRows = 32 / kPieces;
  constexpr int es = OUT_F32 ? 4 : 2;
  const int pc = lane % kPieces;
#pragma unroll
  for (int pass = 0; pass < 32 / kRows; ++pass) {
    const int r = pass * kRows + lane / kPieces;
    dst.u[pass] = (r < rows_valid)
                      ? *reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(base) +
                                                        (elem_off + static_cast<int64_t>(r) * ldc) * es + pc * 16)
                      : make_uint4(0u, 0u, 0u, 0u);
  }
}

// Regroups a block from c_block_load through a staging slot so that lane L
// holds row L (32 values), the layout of the accumulator rows.
template <bool OUT_F32>
__device__ __forceinline__ void c_block_to_row(const CRow<OUT_F32>& blk, uint8_t* slot, int lane, CRow<OUT_F32>& row) {
  constexpr int kPieces = OUT_F32 ? 8 : 4;
  constexpr int kRows = 32 / kPieces;
  const int pc = lane % kPieces;
#pragma unroll
  for (int pass = 0; pass < 32 / kRows; ++pass)
    *reinterpret_cast<uint4*>(slot + stage_off<OUT_F32>(static_cast<uint32_t>(pass * kRows + lane / kPieces), 16u * pc)) =
        blk.u[pass];
  __syncwarp();
#pragma unroll
  for (int k = 0; k < kPieces; ++k)
    row.u[k] = *reinterpret_cast<const uint4*>(slot + stage_off<OUT_F32>(static_cast<uint32_t>(lane), 16u * k));
}

// The 16-bit C block of rows [r0, r0 + 32) and 32 columns, copied with cp.async
// into a staging-layout slot (the access pattern of c_block_load); rows at or
// past `rows_valid` are zero-filled. Completion: cp_async_wait_* + __syncwarp.
__device__ __forceinline__ void c_block_async(uint8_t* slot, const void* base, int64_t elem_off, int64_t ldc,
                                              int rows_valid, int lane) {
  const int pc = lane % 4;
#pragma unroll
  for (int pass = 0; pass < 4; ++pass) {
    const int r = pass * 8 + lane / 4;
    uint8_t* dst = slot + stage_off<false>(static_cast<uint32_t>(r), 16u * pc);
    if (r < rows_valid)
      cp_async_16(dst, static_cast<const uint8_t*>(base) + (elem_off + static_cast<int64_t>(r) * ldc) * 2 + pc * 16, 16);
    else
      cp_async_16(dst, base, 0);
  }
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

// Writes one whole 32 x 32 result block from its staging slots with 16-byte
// stores, each instruction covering 8 rows of 64 bytes (16-bit) or 4 rows of
// 128 bytes (fp32). `buf` holds the block row-major, `tbuf` its transpose:
//   off-diagonal block: D[r0 + r][c0 + c] = buf[r][c]; mirrored (symmetric
//     products): D[c0 + r][r0 + c] = tbuf[r][c]
//   diagonal block: D[r0 + r][r0 + c] = buf[r][c] for c >= r, else tbuf[r][c]
//     (the upper triangle reflected, so the stored block is exactly symmetric)
// D2, when present, receives the same values plus gamma2 on the matrix
// diagonal (`on_diag`: the block holds it).
template <bool OUT_F32>
__device__ __forceinline__ void store_block(const uint8_t* buf, const uint8_t* tbuf, bool diag, bool mirror,
                                            bool on_diag, const GemmEpilogue& epi, int b, int r0, int c0, int lane) {
  constexpr int kPieces = OUT_F32 ? 8 : 4;  // 16-byte pieces per staged row
  constexpr int kElems = OUT_F32 ? 4 : 8;   // elements per piece
  constexpr int kRows = 32 / kPieces;       // rows per instruction
  constexpr int es = OUT_F32 ? 4 : 2;
  const int pc = lane % kPieces;
  uint8_t* d = static_cast<uint8_t*>(epi.d) + (static_cast<int64_t>(b) * epi.d_bstride) * es;
  uint8_t* d2 = epi.has_d2 ? static_cast<uint8_t*>(epi.d2) + (static_cast<int64_t>(b) * epi.d2_bstride) * es : nullptr;
#pragma unroll
  for (int pass = 0; pass < 32 / kRows; ++pass) {
    const int r = pass * kRows + lane / kPieces;
    const uint32_t off = stage_off<OUT_F32>(static_cast<uint32_t>(r), 16u * pc);
    uint4 v = *reinterpret_cast<const uint4*>(buf + off);
    if (diag || mirror) {
      const uint4 t = *reinterpret_cast<const uint4*>(tbuf + off);
      if (mirror) {
        const int64_t row = c0 + r, col = r0 + pc * kElems;
        *reinterpret_cast<uint4*>(d + (row * epi.ldd + col) * es) = t;
        if (d2) *reinterpret_cast<uint4*>(d2 + (row * epi.ldd2 + col) * es) = t;
      } else {
        // Lower-triangle elements (column < row) come from the transpose.
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
        const uint32_t tw[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int e = 0; e < kElems; ++e) {
          const int c = pc * kElems + e;
          if (c >= r) continue;
          if (OUT_F32) {
            w[e] = tw[e];
          } else {
            const uint32_t mask = (e & 1) ? 0xffff0000u : 0x0000ffffu;
            w[e >> 1] = (w[e >> 1] & ~mask) | (tw[e >> 1] & mask);
          }
        }
        v = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    const int64_t row = r0 + r, col = c0 + pc * kElems;
    *reinterpret_cast<uint4*>(d + (row * epi.ldd + col) * es) = v;
    if (d2) {
      uint4 v2 = v;
      if (on_diag && r / kElems == pc) {
        // gamma2 on the element at column r of this row.
        uint32_t w[4] = {v2.x, v2.y, v2.z, v2.w};
#pragma unroll
        for (int e = 0; e < kElems; ++e) {
          if (pc * kElems + e != r) continue;
          if (OUT_F32) {
            w[e] = __float_as_uint(__uint_as_float(w[e]) + epi.gamma2);
          } else {
            const uint32_t sh = (e & 1) ? 16u : 0u;
            const uint16_t h = static_cast<uint16_t>(w[e >> 1] >> sh);
            const uint32_t nh = float_to_half_bits(half_bits_to_float(h, epi.out_bf16) + epi.gamma2, epi.out_bf16);
            w[e >> 1] = (w[e >> 1] & ~(0xffffu << sh)) | (nh << sh);
          }
        }
        v2 = make_uint4(w[0], w[1], w[2], w[3]);
      }
      *reinterpret_cast<uint4*>(d2 + (row * epi.ldd2 + col) * es) = v2;
    }
  }
}

// Number of leading k-blocks of a tile whose rows start at `row0` that lie below
// the block diagonal of an upper-stored symmetric operand (read transposed).
__device__ __forceinline__ int upper_kblocks(int upper, int row0, int k_blocks) {
  if (!upper) return 0;
  const int n = (row0 / kUpperBlock) * (kUpperBlock / kBK);
  return n < k_blocks ? n : k_blocks;
}

// UP: operands may be upper-stored symmetric matrices (GemmShape::a_upper /
// b_upper); instantiated only for the chains' layouts, so other launches carry
// no per-k-block checks on the producer and MMA paths.
template <int BN, bool A_MN, bool B_MN, bool OUT_F32, bool SYM, bool PAIR, bool UP>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_at, const __grid_constant__ CUtensorMap tmap_bt,
                   const GemmShape shape, const GemmEpilogue epi,
                   const int ab_bf16) {
  using Cfg = GemmConfig<BN, OUT_F32, PAIR>;
  constexpr int S = Cfg::kStages;
  constexpr uint32_t CB = Cfg::kChunkBytes;
  constexpr int kTileM = Cfg::kTileM;
  // Pair mode: CTA 0 issues the MMAs and owns the full and accumulator-empty
  // barriers; both CTAs load, and both run an epilogue over their own TMEM rows.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int tile_first = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int tile_step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + S * Cfg::kABytes;
  uint8_t* smem_epi = smem + S * Cfg::kStageBytes;
  uint8_t* smem_cring = smem_epi + Cfg::kEpiBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_cring + Cfg::kCRingBytes);
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
      mbar_init(&tempty_bar[a], (PAIR ? 2 : 1) * kEpiWarps);  // one arrival per epilogue warp
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
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (PAIR)
    cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Set-up above overlaps the previous kernel's tail; operands and C are read below.
  pdl_launch_dependents();
  pdl_wait_predecessor();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      // Pair mode: the bytes of both CTAs complete on CTA 0's full barrier.
      const uint32_t full0 = PAIR ? cluster_addr(&full_bar[0], 0) : 0u;
      for (int t = tile_first; t < shape.total_tiles; t += tile_step) {
        int b, i, j;
        decode_tile<BN, SYM, kTileM>(shape, t, b, i, j);
        const int m0 = i * kTileM + static_cast<int>(rank) * kBM;
        const int n0 = j * BN + static_cast<int>(rank) * Cfg::kBRows;
        // Upper-stored symmetric operands: the first kb_a (kb_b) k-blocks of the
        // tile lie below the block diagonal and come transposed.
        const int kb_a = UP ? upper_kblocks(shape.a_upper, i * kTileM, shape.k_blocks) : 0;
        const int kb_b = UP ? upper_kblocks(shape.b_upper, j * BN, shape.k_blocks) : 0;
        for (int kb = 0; kb < shape.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[st], ph ^ 1u, abort_flag, &g_device_status, kStatusProducerTimeout))
            goto producer_done;
          const int k0 = kb * kBK;
          uint8_t* sa = smem_a + st * Cfg::kABytes;
          uint8_t* sb = smem_b + st * Cfg::kBBytes;
          const bool a_mn = A_MN || (UP && kb < kb_a);
          const bool b_mn = B_MN || (UP && kb < kb_b);
          const CUtensorMap* ma = (!UP || A_MN || !a_mn) ? &tmap_a : &tmap_at;
          const CUtensorMap* mb = (!UP || B_MN || !b_mn) ? &tmap_b : &tmap_bt;
          if (PAIR) {
            if (rank == 0) mbar_arrive_expect_tx(&full_bar[st], 2 * Cfg::kStageBytes);
            const uint32_t fb = full0 + static_cast<uint32_t>(st) * 8u;
            if (!a_mn) {
              tma_load_3d_pair(sa, ma, fb, k0, m0, b);
            } else {
#pragma unroll
              for (int ch = 0; ch < kBM / 64; ++ch) tma_load_3d_pair(sa + ch * 8192, ma, fb, m0 + 64 * ch, k0, b);
            }
            if (!b_mn) {
              tma_load_3d_pair(sb, mb, fb, k0, n0, b);
            } else {
#pragma unroll
              for (int ch = 0; ch < Cfg::kBRows / 64; ++ch) tma_load_3d_pair(sb + ch * 8192, mb, fb, n0 + 64 * ch, k0, b);
            }
          } else {
            mbar_arrive_expect_tx(&full_bar[st], Cfg::kStageBytes);
            if (!a_mn) {
              tma_load_3d(sa, ma, &full_bar[st], k0, m0, b);
            } else {
#pragma unroll
              for (int ch = 0; ch < kBM / 64; ++ch) tma_load_3d(sa + ch * 8192, ma, &full_bar[st], m0 + 64 * ch, k0, b);
            }
            if (!b_mn) {
              tma_load_3d(sb, mb, &full_bar[st], k0, n0, b);
            } else {
#pragma unroll
              for (int ch = 0; ch < BN / 64; ++ch) tma_load_3d(sb + ch * 8192, mb, &full_bar[st], n0 + 64 * ch, k0, b);
            }
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
    if (lane == 0 && rank == 0) {
      // One instruction descriptor per operand-major combination (upper-stored
      // symmetric operands switch to MN-major below the block diagonal).
      const uint32_t idesc_kk = make_idesc_f16(ab_bf16, A_MN ? 1 : 0, B_MN ? 1 : 0, kTileM, BN);
      const uint32_t idesc_tk = make_idesc_f16(ab_bf16, 1, B_MN ? 1 : 0, kTileM, BN);
      const uint32_t idesc_kt = make_idesc_f16(ab_bf16, A_MN ? 1 : 0, 1, kTileM, BN);
      const uint32_t idesc_tt = make_idesc_f16(ab_bf16, 1, 1, kTileM, BN);
      // Shared-memory descriptors of a stage: K-major tiles advance 32 bytes per
      // K=16 step and MN-major tiles 2 KB, i.e. 2 or 128 in the descriptor's
      // start-address field (bytes >> 4; shared memory stays below 256 KB, so
      // the 14-bit field never carries).
      const uint64_t desc_k = make_smem_desc_sw128(0, 16, 1024);
      const uint64_t desc_t = make_smem_desc_sw128(0, 8192, 1024);
      // Pair mode: completions are signalled to the barrier at the same offset in both CTAs.
      const uint32_t empty0 = PAIR ? cluster_addr(&empty_bar[0], 0) : 0u;
      const uint32_t empty1 = PAIR ? cluster_addr(&empty_bar[0], 1) : 0u;
      const uint32_t tfull0 = PAIR ? cluster_addr(&tfull_bar[0], 0) : 0u;
      const uint32_t tfull1 = PAIR ? cluster_addr(&tfull_bar[0], 1) : 0u;
      int st = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      for (int t = tile_first; t < shape.total_tiles; t += tile_step) {
        int kb_a = 0, kb_b = 0;
        if (UP) {
          int tb, ti, tj;
          decode_tile<BN, SYM, kTileM>(shape, t, tb, ti, tj);
          kb_a = upper_kblocks(shape.a_upper, ti * kTileM, shape.k_blocks);
          kb_b = upper_kblocks(shape.b_upper, tj * BN, shape.k_blocks);
        }
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
          const uint64_t a_addr = static_cast<uint64_t>((smem_u32(smem_a + st * Cfg::kABytes) >> 4) & 0x3FFFu);
          const uint64_t b_addr = static_cast<uint64_t>((smem_u32(smem_b + st * Cfg::kBBytes) >> 4) & 0x3FFFu);
          const bool a_mn = A_MN || (UP && kb < kb_a);
          const bool b_mn = B_MN || (UP && kb < kb_b);
          const uint32_t idesc = !UP ? idesc_kk : (a_mn ? (b_mn ? idesc_tt : idesc_tk) : (b_mn ? idesc_kt : idesc_kk));
          // K-major: advance 16 elements (32 bytes) inside the swizzle row.
          // MN-major: advance 16 K-rows (2 x 1024-byte swizzle atoms); LBO = 8 KB chunk stride.
          const uint64_t adesc0 = (a_mn ? desc_t : desc_k) + a_addr;
          const uint64_t bdesc0 = (b_mn ? desc_t : desc_k) + b_addr;
          const uint32_t a_step = a_mn ? 128u : 2u, b_step = b_mn ? 128u : 2u;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t adesc = adesc0 + kk * a_step;
            const uint64_t bdesc = bdesc0 + kk * b_step;
            if (PAIR)
              tc_mma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            else
              tc_mma_f16(d_tmem, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          if (PAIR) {
            tc_commit_pair(empty0 + static_cast<uint32_t>(st) * 8u);
            tc_commit_pair(empty1 + static_cast<uint32_t>(st) * 8u);
          } else {
            tc_commit(&empty_bar[st]);
          }
          if (++st == S) {
            st = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        if (PAIR) {
          tc_commit_pair(tfull0 + static_cast<uint32_t>(acc) * 8u);
          tc_commit_pair(tfull1 + static_cast<uint32_t>(acc) * 8u);
        } else {
          tc_commit(&tfull_bar[acc]);
        }
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1u;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Each warp owns two staging slots: a result block and its transpose.
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const int half = ew >> 2;      // even (0) or odd (1) 32-column chunks
    uint8_t* ring = smem_epi + ew * kRing * CB;
    const int bf16 = epi.out_bf16;
    const bool use_c = epi.has_c != 0;
    constexpr int kChunks = BN / 32;
    constexpr bool CR = Cfg::kCRing;
    uint8_t* cring = smem_cring + (CR ? ew * 2 * CB : 0u);
    constexpr int kCDepth = (OUT_F32 || CR) ? 1 : 2;  // C blocks held in registers per warp
    int acc = 0;
    uint32_t acc_ph = 0;
    bool aborted = false;

    const uint32_t tempty0 = PAIR ? cluster_addr(&tempty_bar[0], 0) : 0u;
    for (int t = tile_first; t < shape.total_tiles && !aborted; t += tile_step) {
      int b, i, j;
      decode_tile<BN, SYM, kTileM>(shape, t, b, i, j);
      const int r0 = i * kTileM + static_cast<int>(rank) * kBM + quarter * 32;
      const int cbase = j * BN;
      // Needed chunks form the run [first, end): in range, and column >= row when symmetric.
      int end = (shape.N - cbase + 31) / 32;
      end = end < kChunks ? end : kChunks;
      // Upper block storage mirrors only inside the diagonal kUpperBlock band (the
      // stored matrix stays exactly symmetric there; outside it the lower blocks
      // are not stored). The tile's 256 columns lie in one block column.
      const bool mirror_band = SYM && (!epi.upper_out || cbase / kUpperBlock == r0 / kUpperBlock);
      int first = mirror_band ? ((r0 > cbase) ? (r0 - cbase) / 32 : 0) : 0;
      if (r0 >= shape.M) first = end;
      // C rows travel through the LSU path (not the TMA queue, where they would
      // wait behind the main loop's operand tiles) into registers.
      const int64_t c_row = static_cast<int64_t>(b) * epi.c_bstride + static_cast<int64_t>(r0 + lane) * epi.ldc;
      // Blocks whose 32 columns are in range and 16-byte aligned load coalesced.
      auto c_ok = [&](int cc) { return use_c && epi.c_vec && (cbase + cc * 32 + 32 <= shape.N); };
      const int64_t c_blk = static_cast<int64_t>(b) * epi.c_bstride + static_cast<int64_t>(r0) * epi.ldc + cbase;
      const int c_rows = shape.M - r0;
      // The first C blocks of this warp are requested before the accumulator is
      // ready, so their latency hides behind the main loop. Ring mode keeps two
      // blocks in flight in shared memory: one cp.async group per block slot,
      // committed even when empty, so "all but the newest group complete" always
      // means the block about to be used has landed.
      CRow<OUT_F32> cq[kCDepth];
      const int start = first + (((first & 1) != half) ? 1 : 0);  // this warp's chunks: start, start + 2, ...
      auto c_ring_issue = [&](uint8_t* slot, int qc) {
        if (qc < end && c_ok(qc)) c_block_async(slot, epi.c, c_blk + qc * 32, epi.ldc, c_rows, lane);
        cp_async_commit();
      };
      int cslot = 0;
      if (CR) {
        if (use_c) {
          c_ring_issue(cring, start);
          c_ring_issue(cring + CB, start + 2);
        }
      } else {
#pragma unroll
        for (int q = 0; q < kCDepth; ++q) {
          const int qc = start + 2 * q;
          if (qc < end && c_ok(qc)) c_block_load<OUT_F32>(cq[q], epi.c, c_blk + qc * 32, epi.ldc, c_rows, lane);
        }
      }
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_ph, abort_flag, &g_device_status, kStatusEpilogueTimeout)) {
        aborted = true;
        break;
      }
      __syncwarp();
      tc_fence_after();
      const uint32_t lane_addr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int cc = start; cc < end; cc += 2) {
        const int c0 = cbase + cc * 32;
        float v[32];
        __syncwarp();
        tmem_load_32cols(lane_addr + cc * 32, v);
        float cv[32];
        if (CR && use_c) {
          cp_async_wait_1();
          __syncwarp();
          uint8_t* cs = cring + cslot * CB;
          if (c_ok(cc)) {
            CRow<OUT_F32> crow;
#pragma unroll
            for (int k = 0; k < (OUT_F32 ? 8 : 4); ++k)
              crow.u[k] = *reinterpret_cast<const uint4*>(cs + stage_off<OUT_F32>(static_cast<uint32_t>(lane), 16u * k));
            c_row_unpack<OUT_F32>(crow, bf16, cv);
          } else {
#pragma unroll
            for (int q = 0; q < 32; ++q)
              cv[q] = (r0 + lane < shape.M && c0 + q < shape.N) ? global_get<OUT_F32>(epi.c, c_row + c0 + q, bf16) : 0.0f;
          }
          __syncwarp();  // every lane has read the slot before it is refilled
          c_ring_issue(cs, cc + 4);
          cslot ^= 1;
        } else if (use_c) {
          if (c_ok(cc)) {
            CRow<OUT_F32> crow;
            c_block_to_row<OUT_F32>(cq[0], ring, lane, crow);
            c_row_unpack<OUT_F32>(crow, bf16, cv);
          } else {
#pragma unroll
            for (int q = 0; q < 32; ++q)
              cv[q] = (r0 + lane < shape.M && c0 + q < shape.N) ? global_get<OUT_F32>(epi.c, c_row + c0 + q, bf16) : 0.0f;
          }
#pragma unroll
          for (int q = 0; q + 1 < kCDepth; ++q) cq[q] = cq[q + 1];
          const int qc = cc + 2 * kCDepth;
          if (qc < end && c_ok(qc)) c_block_load<OUT_F32>(cq[kCDepth - 1], epi.c, c_blk + qc * 32, epi.ldc, c_rows, lane);
        }
        XRow<OUT_F32> x;
        if (!OUT_F32 && (epi.round_dtype < 0 || (epi.round_dtype == kF16 && bf16))) {
          // 16-bit output (optionally rounded through fp16 first): paired conversions.
          const bool via_f16 = epi.round_dtype == kF16;
#pragma unroll
          for (int q = 0; q < 32; q += 2) {
            float y0 = epi.alpha * v[q], y1 = epi.alpha * v[q + 1];
            if (use_c) {
              y0 = fmaf(epi.beta, cv[q], y0);
              y1 = fmaf(epi.beta, cv[q + 1], y1);
            }
            if (via_f16) {
              const float2 r = __half22float2(__floats2half2_rn(y0, y1));
              y0 = r.x;
              y1 = r.y;
            }
            x.w[q >> 1] = pack_pair(y0, y1, bf16);
          }
        } else {
#pragma unroll
          for (int q = 0; q < 32; ++q) {
            float y = epi.alpha * v[q];
            if (use_c) y = fmaf(epi.beta, cv[q], y);
            if (epi.round_dtype >= 0) y = round_to(y, epi.round_dtype);
            if (OUT_F32) {
              x.w[q] = __float_as_uint(y);
            } else {
              const uint32_t h = float_to_half_bits(y, bf16);
              x.w[q >> 1] = (q & 1) ? (x.w[q >> 1] | (h << 16)) : h;
            }
          }
        }
        const bool on_diag = SYM && (c0 == r0);  // holds the matrix diagonal (gamma2 of D2)
        // Symmetrise diagonal blocks and mirror the other blocks of the band
        // (full storage: the whole matrix is the band).
        const bool diag = on_diag;
        const bool mirror = mirror_band && !on_diag;
        // The block goes to slot 0 row-major and, in symmetric mode, to slot 1
        // transposed (slot 1 row q holds column q of the block).
        uint8_t* buf = ring;
        uint8_t* tbuf = ring + CB;
        __syncwarp();  // every lane is done with the previous block's slots
        stage_write_row<OUT_F32>(buf, lane, x);
        if (diag || mirror) stage_write_col<OUT_F32>(tbuf, lane, x);
        __syncwarp();
        // Whole blocks with 16-byte aligned rows: coalesced vector stores (the
        // mirror block of a symmetric product is whole too, since M == N there).
        const bool vec = epi.vec_d && (!epi.has_d2 || epi.vec_d2) && (r0 + 32 <= shape.M) && (c0 + 32 <= shape.N);
        if (vec) {
          store_block<OUT_F32>(buf, tbuf, diag, mirror, on_diag, epi, b, r0, c0, lane);
        } else {
          // Generic path: blocks on the matrix edge and outputs whose rows are not
          // 16-byte aligned. Lane = column, loop = row: coalesced rows.
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
            // Strictly upper block on the edge or with unaligned rows:
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
        }
      }
      if (aborted) break;
      // Every lane's TMEM reads are complete (tcgen05.wait::ld); one arrival per warp
      // releases the accumulator buffer (CTA 0's barrier in pair mode).
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR)
          mbar_arrive_cluster(tempty0 + static_cast<uint32_t>(acc) * 8u);
        else
          mbar_arrive(&tempty_bar[acc]);
      }
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1u;
    }
    if (CR) cp_async_wait_all();  // no copy may land after the CTA's shared memory is released
  }

  // Teardown: all roles meet; on abort give in-flight TMA/MMA work time to land
  // before TMEM and shared memory are released.
  // In pair mode neither CTA leaves while the other may still signal its
  // barriers or while CTA 0's MMAs may still write its TMEM.
  tc_fence_before();
  if (PAIR)
    cluster_sync_all();
  else
    __syncthreads();
  if (*abort_flag) settle_for_ns(2000000ull);
  if (PAIR)
    cluster_sync_all();
  else
    __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    else
      tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace gns
