// Fused Gram Newton-Schulz chain for matrices whose short side m is at most 128.
//
// The multi-launch chain (ns_chain.cu) runs one tcgen05 GEMM launch per
// product: 18 launches for five iterations with one reset. For small matrices
// each launch does well under a microsecond of tensor work but costs several
// microseconds of launch, set-up and pipeline fill, so the chain is latency
// bound. Here ONE CTA runs the whole chain of one matrix (persistently, over
// the batch):
//
//   G = X X^T  ->  Gram-space products (newton_schulz.py:177-212)
//   -> X <- Q X at a reset, G rebuilt (:164-175)  ->  O = Q X
//
// G, P, GP and Q stay in shared memory as fp16 128 x 128 matrices in the
// tensor core's 128-byte-swizzled K-major layout, so the Gram-space products
// read their operands and accumulator inputs from shared memory and write
// their results back there: they never touch global memory. X streams through
// a ring of four 16 KB TMA slots. The accumulators are two 128-column TMEM
// buffers, so the epilogue of one X-product tile overlaps the next tile's MMAs.
//
// Roles (320 threads):
//   warp 0      TMA producer (lane 0)
//   warp 1      TMEM allocator + MMA issuer (lane 0)
//   warps 2..9  epilogue: two 32 x 32 blocks of each 128 x 128 result per warp
//               (warp w reads TMEM lanes 32 (w mod 4) .. +31)
// All three roles walk the same sequence of units (walk_chain) and meet on
// mbarriers:
//   full/empty   slot ring between producer and MMA
//   tfull/tempty accumulator buffers between MMA and epilogue
//   opnd         the epilogue finished a shared-memory matrix (the next
//                product may read it)
//   xready       the epilogue finished writing the reset X to global memory
//                (the producer may load it for the next Gram matrix)
//   ebar         epilogue-only barrier (every warp's stores of a matrix landed)
//
// Arithmetic equals the multi-launch chain's: the same MMA shapes along K (16
// per instruction, in order), alpha * acc + beta * C with one fma, fp16
// rounding of every Gram-space matrix, the lower triangle of every symmetric
// product copied from its upper triangle, and Q = P + a I formed from the
// rounded P. Every wait is bounded (gns_common.cuh); on expiry the kernel
// records a status code, lets in-flight work land, frees TMEM and returns.
#include <atomic>
#include <mutex>

#include "../../include/gns_b200.h"
#include "gns_common.cuh"
#include "gns_host.h"

namespace gns {

// Set by a small-chain CTA whose bounded wait gave up; read by gns_device_status().
__device__ int g_small_chain_status = 0;

namespace {

constexpr int kSmallM = 128;  // largest short side
// Longest long side routed here. One CTA streams its matrix's whole long side,
// while the multi-launch chain spreads each product over every SM, so past a
// few thousand columns the multi-launch chain wins at every batch size.
// Measured on B200 (bf16, short side 128, fused vs multi-launch): n = 2048
// 114 vs 143 us; n = 4096 179 vs 162 us at batch 1 and 186 vs 181 us at
// batch 16; n = 8192 418 vs 397 us at batch 64.
constexpr int64_t kSmallMaxN = 3072;
constexpr int kSlots = 4;
constexpr uint32_t kSlotBytes = 16384;    // 128 x 64 fp16: one k-block of a 128-row tile
constexpr uint32_t kMatBytes = 32768;     // 128 x 128 fp16
constexpr int kMats = 4;
constexpr int kEpiWarpsSC = 8;
constexpr int kThreadsSC = 32 * (2 + kEpiWarpsSC);
constexpr uint32_t kAccCols = 128;
constexpr uint32_t kTmemColsSC = 2 * kAccCols;
constexpr int kBarCount = 2 * kSlots + 4 + 4;
constexpr size_t kSmemBytesSC = 1024 + kSlots * kSlotBytes + kMats * kMatBytes + kBarCount * 8 + 16;
constexpr int kMaxItersSC = 32;

enum Mat : int { kMatG = 0, kMatP = 1, kMatGP = 2, kMatQ = 3, kNone = -1 };
// The square (standard) chain keeps X where the Gram chain keeps GP.
constexpr int kMatX = kMatGP;
enum Mode : int { kWide = 0, kTall = 1, kSquare = 2 };

struct SmallChainParams {
  int batch, m, n;
  int n_iters;
  uint32_t reset_mask;
  float coef[kMaxItersSC][3];  // (a, b, c) per iteration, as the multi-launch chain rounds them
  __half* x[2];                // normalised X and the reset buffer, [batch][rows][ldx]
  int64_t ldx, xb;
  void* out;
  int out_dtype;
  int64_t out_bstride, out_rstride;
  int out_vec;  // output base and row/batch strides 16-byte aligned
  int x_vec;    // X buffers' rows 16-byte aligned
};

// Byte offset of element (r, c) of a 128 x 128 fp16 matrix in the 128-byte
// swizzled K-major layout: two 16 KB atoms of 64 columns; row r at 128 r; the
// 16-byte chunk j of a row stored at position j ^ (r mod 8). This is the layout
// a TMA SWIZZLE_128B load of 64 x 64 boxes produces and the layout the MMA's
// shared-memory descriptors (SBO = 1024) describe.
__device__ __forceinline__ uint32_t mat_off(uint32_t r, uint32_t c) {
  return ((c >> 6) << 14) + (r << 7) + ((((c >> 3) & 7u) ^ (r & 7u)) << 4) + ((c & 7u) << 1);
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// The unit sequence of one matrix, shared by all roles. Each visitor call
// returns false when the CTA aborts.
template <class V>
__device__ __forceinline__ bool walk_chain(const SmallChainParams& p, V& v) {
  int xi = 0;
  if (!v.gram(xi)) return false;
  int begin = 0;
  for (int it = 1; it <= p.n_iters; ++it) {
    if (it < p.n_iters && !((p.reset_mask >> it) & 1u)) continue;
    bool have_q = false;
    for (int j = begin; j < it; ++j) {
      const float a = p.coef[j][0], bq = p.coef[j][1], c = p.coef[j][2];
      if (!have_q) {
        // P = c G^2 + b G and Q = P + a I.
        if (!v.sym(kMatG, kMatG, kMatG, c, bq, kMatP, kMatQ, a)) return false;
        have_q = true;
      } else {
        if (!v.sym(kMatG, kMatG, kMatG, c, bq, kMatP, kNone, 0.0f)) return false;
        // Q <- Q P + a Q (in place: the MMAs finish reading Q before the epilogue writes it).
        if (!v.sym(kMatQ, kMatP, kMatQ, 1.0f, a, kMatQ, kNone, 0.0f)) return false;
      }
      if (j + 1 < it) {
        if (!v.sym(kMatG, kMatP, kMatG, 1.0f, a, kMatGP, kNone, 0.0f)) return false;
        if (!v.sym(kMatP, kMatGP, kMatGP, 1.0f, a, kMatG, kNone, 0.0f)) return false;
      }
    }
    if (it < p.n_iters) {
      if (!v.xprod(xi, true)) return false;
      xi ^= 1;
      if (!v.gram(xi)) return false;
    }
    begin = it;
  }
  return v.xprod(xi, false);
}

// Standard Newton-Schulz on a square matrix (newton_schulz.py:66-121): per
// iteration G = X X^T, P = c G^2 + b G, X <- P X + a X; the last X goes out.
template <class V>
__device__ __forceinline__ bool walk_standard(const SmallChainParams& p, V& v) {
  for (int it = 0; it < p.n_iters; ++it) {
    const float a = p.coef[it][0], bq = p.coef[it][1], c = p.coef[it][2];
    if (!v.square_gram(it == 0)) return false;
    if (!v.sym(kMatG, kMatG, kMatG, c, bq, kMatP, kNone, 0.0f)) return false;
    if (!v.square_xprod(a, it + 1 == p.n_iters)) return false;
  }
  return true;
}

struct Shared {
  uint8_t* slots;
  uint8_t* mats;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* tfull;
  uint64_t* tempty;
  uint64_t* opnd;
  uint64_t* xready;
  uint64_t* ebar;
  uint64_t* xload;  // square chain: the TMA load of X into shared memory
  volatile int* abort_flag;
};

template <bool TALL>
struct ProducerRole {
  const SmallChainParams& p;
  const Shared s;
  const CUtensorMap* map0;
  const CUtensorMap* map1;
  int b = 0;
  int st = 0;
  uint32_t ph = 0, xr_ph = 0;

  __device__ ProducerRole(const SmallChainParams& p_, const Shared& s_, const CUtensorMap* m0, const CUtensorMap* m1)
      : p(p_), s(s_), map0(m0), map1(m1) {}

  __device__ bool slot(uint8_t*& dst, uint64_t*& bar) {
    if (!mbar_wait_bounded(&s.empty[st], ph ^ 1u, s.abort_flag, &g_small_chain_status, kStatusProducerTimeout))
      return false;
    mbar_arrive_expect_tx(&s.full[st], kSlotBytes);
    dst = s.slots + st * kSlotBytes;
    bar = &s.full[st];
    if (++st == kSlots) {
      st = 0;
      ph ^= 1u;
    }
    return true;
  }

  // Gram k-blocks: 64 columns of X (wide: the 128 rows as two 64-row boxes,
  // K-major; tall: 64 rows of X as two 64-column boxes, MN-major).
  __device__ bool gram(int xi) {
    const CUtensorMap* map = xi ? map1 : map0;
    const int kbn = (p.n + 63) / 64;
    for (int kb = 0; kb < kbn; ++kb) {
      uint8_t* d;
      uint64_t* bar;
      if (!slot(d, bar)) return false;
      if (!TALL) {
        tma_load_3d(d, map, bar, kb * 64, 0, b);
        tma_load_3d(d + 8192, map, bar, kb * 64, 64, b);
      } else {
        tma_load_3d(d, map, bar, 0, kb * 64, b);
        tma_load_3d(d + 8192, map, bar, 64, kb * 64, b);
      }
    }
    return true;
  }

  __device__ bool sym(int, int, int, float, float, int, int, float) { return true; }

  // Square chain: X (m x m, at most 128 x 128) into its shared-memory matrix as
  // four 64 x 64 boxes, once the previous matrix's last product released it.
  int loaded = 0;
  __device__ bool square_gram(bool first) {
    if (!first) return true;
    if (loaded > 0) {
      if (!mbar_wait_bounded(s.xready, xr_ph, s.abort_flag, &g_small_chain_status, kStatusProducerTimeout))
        return false;
      xr_ph ^= 1u;
    }
    ++loaded;
    uint8_t* xm = s.mats + kMatX * kMatBytes;
    mbar_arrive_expect_tx(s.xload, kMatBytes);
    tma_load_3d(xm, map0, s.xload, 0, 0, b);
    tma_load_3d(xm + 8192, map0, s.xload, 0, 64, b);
    tma_load_3d(xm + 16384, map0, s.xload, 64, 0, b);
    tma_load_3d(xm + 24576, map0, s.xload, 64, 64, b);
    return true;
  }

  __device__ bool square_xprod(float, bool) { return true; }

  // X-product tiles of 128 along the long side, k-blocks of 64 along m.
  __device__ bool xprod(int xi, bool reset) {
    const CUtensorMap* map = xi ? map1 : map0;
    const int tiles = (p.n + 127) / 128, kbm = (p.m + 63) / 64;
    for (int t = 0; t < tiles; ++t) {
      for (int kb = 0; kb < kbm; ++kb) {
        uint8_t* d;
        uint64_t* bar;
        if (!slot(d, bar)) return false;
        if (!TALL) {
          tma_load_3d(d, map, bar, t * 128, kb * 64, b);
          tma_load_3d(d + 8192, map, bar, t * 128 + 64, kb * 64, b);
        } else {
          tma_load_3d(d, map, bar, kb * 64, t * 128, b);
          tma_load_3d(d + 8192, map, bar, kb * 64, t * 128 + 64, b);
        }
      }
    }
    if (reset) {
      // The next Gram matrix reads the reset X: wait until the epilogue wrote it.
      if (!mbar_wait_bounded(s.xready, xr_ph, s.abort_flag, &g_small_chain_status, kStatusProducerTimeout))
        return false;
      xr_ph ^= 1u;
    }
    return true;
  }
};

template <bool TALL>
struct MmaRole {
  const SmallChainParams& p;
  const Shared s;
  uint32_t tmem_base;
  int st = 0;
  uint32_t ph = 0;
  int acc = 0;
  uint32_t acc_ph = 0;
  uint32_t opnd_ph = 0;
  uint32_t xl_ph = 0;
  uint64_t desc_k, desc_t, desc_xmn;
  uint32_t idesc_gram, idesc_sym, idesc_x, idesc_sqx;

  __device__ MmaRole(const SmallChainParams& p_, const Shared& s_, uint32_t tmem)
      : p(p_), s(s_), tmem_base(tmem) {
    desc_k = make_smem_desc_sw128(0, 16, 1024);    // K-major: 8-row groups 1 KB apart
    desc_t = make_smem_desc_sw128(0, 8192, 1024);  // MN-major: 64-wide chunks 8 KB apart
    idesc_gram = make_idesc_f16(0, TALL ? 1 : 0, TALL ? 1 : 0, 128, 128);
    idesc_sym = make_idesc_f16(0, 0, 0, 128, 128);
    idesc_x = make_idesc_f16(0, 0, TALL ? 0 : 1, 128, 128);
    desc_xmn = make_smem_desc_sw128(0, 16384, 1024);  // a 128 x 128 matrix read MN-major
    idesc_sqx = make_idesc_f16(0, 0, 1, 128, 128);
  }

  __device__ uint64_t slot_desc(uint64_t base) const {
    return base + static_cast<uint64_t>((smem_u32(s.slots + st * kSlotBytes) >> 4) & 0x3FFFu);
  }

  // Descriptor of K-step kk (16 columns) of a shared-memory matrix.
  __device__ uint64_t mat_desc(int mat, int kk) const {
    const uint32_t addr = smem_u32(s.mats + mat * kMatBytes) + (kk >> 2) * 16384u + (kk & 3) * 32u;
    return desc_k + static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  }

  __device__ bool take_acc(uint32_t& d) {
    if (!mbar_wait_bounded(&s.tempty[acc], acc_ph ^ 1u, s.abort_flag, &g_small_chain_status, kStatusMmaTimeout))
      return false;
    tc_fence_after();
    d = tmem_base + static_cast<uint32_t>(acc) * kAccCols;
    return true;
  }

  __device__ void give_acc() {
    tc_commit(&s.tfull[acc]);
    acc ^= 1;
    if (acc == 0) acc_ph ^= 1u;
  }

  __device__ bool wait_full() {
    if (!mbar_wait_bounded(&s.full[st], ph, s.abort_flag, &g_small_chain_status, kStatusMmaTimeout)) return false;
    tc_fence_after();
    return true;
  }

  __device__ void free_slot() {
    tc_commit(&s.empty[st]);
    if (++st == kSlots) {
      st = 0;
      ph ^= 1u;
    }
  }

  __device__ bool wait_operands() {
    if (!mbar_wait_bounded(s.opnd, opnd_ph, s.abort_flag, &g_small_chain_status, kStatusMmaTimeout)) return false;
    opnd_ph ^= 1u;
    tc_fence_after();
    return true;
  }

  __device__ bool gram(int) {
    uint32_t d;
    if (!take_acc(d)) return false;
    const int kbn = (p.n + 63) / 64;
    for (int kb = 0; kb < kbn; ++kb) {
      if (!wait_full()) return false;
      const uint64_t base = slot_desc(TALL ? desc_t : desc_k);
      const uint32_t step = TALL ? 128u : 2u;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        tc_mma_f16(d, base + kk * step, base + kk * step, idesc_gram, (kb > 0 || kk > 0) ? 1u : 0u);
      free_slot();
    }
    give_acc();
    return true;
  }

  __device__ bool sym(int A, int B, int, float, float, int, int, float) {
    if (!wait_operands()) return false;
    uint32_t d;
    if (!take_acc(d)) return false;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) tc_mma_f16(d, mat_desc(A, kk), mat_desc(B, kk), idesc_sym, kk > 0 ? 1u : 0u);
    give_acc();
    return true;
  }

  // Square chain. Gram: A = B = X (rows, K-major).
  __device__ bool square_gram(bool first) {
    if (first) {
      if (!mbar_wait_bounded(s.xload, xl_ph, s.abort_flag, &g_small_chain_status, kStatusMmaTimeout)) return false;
      xl_ph ^= 1u;
      tc_fence_after();
    } else if (!wait_operands()) {
      return false;
    }
    uint32_t d;
    if (!take_acc(d)) return false;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      tc_mma_f16(d, mat_desc(kMatX, kk), mat_desc(kMatX, kk), idesc_sym, kk > 0 ? 1u : 0u);
    give_acc();
    return true;
  }

  // Square chain: P X with X read MN-major (its 64-column atoms 16 KB apart, 16 rows per K step).
  __device__ bool square_xprod(float, bool) {
    if (!wait_operands()) return false;
    uint32_t d;
    if (!take_acc(d)) return false;
    const uint32_t xbase = smem_u32(s.mats + kMatX * kMatBytes);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      tc_mma_f16(d, mat_desc(kMatP, kk), desc_xmn + static_cast<uint64_t>(((xbase + kk * 2048u) >> 4) & 0x3FFFu),
                 idesc_sqx, kk > 0 ? 1u : 0u);
    give_acc();
    return true;
  }

  __device__ bool xprod(int, bool) {
    if (!wait_operands()) return false;
    const int tiles = (p.n + 127) / 128, kbm = (p.m + 63) / 64;
    for (int t = 0; t < tiles; ++t) {
      uint32_t d;
      if (!take_acc(d)) return false;
      for (int kb = 0; kb < kbm; ++kb) {
        if (!wait_full()) return false;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t acc_flag = (kb > 0 || kk > 0) ? 1u : 0u;
          if (!TALL)  // Q (K-major) times X (MN-major)
            tc_mma_f16(d, mat_desc(kMatQ, 4 * kb + kk), slot_desc(desc_t) + kk * 128u, idesc_x, acc_flag);
          else  // X rows (K-major) times Q
            tc_mma_f16(d, slot_desc(desc_k) + kk * 2u, mat_desc(kMatQ, 4 * kb + kk), idesc_x, acc_flag);
        }
        free_slot();
      }
      give_acc();
    }
    return true;
  }
};

template <bool TALL>
struct EpilogueRole {
  const SmallChainParams& p;
  const Shared s;
  uint32_t tmem_base;
  int b = 0;
  int lane, quarter, half;
  int acc = 0;
  uint32_t acc_ph = 0;
  uint32_t e_ph = 0;

  __device__ EpilogueRole(const SmallChainParams& p_, const Shared& s_, uint32_t tmem, int warp, int lane_)
      : p(p_), s(s_), tmem_base(tmem), lane(lane_) {
    quarter = warp & 3;
    half = (warp - 2) >> 2;
  }

  __device__ bool wait_acc() {
    if (!mbar_wait_bounded(&s.tfull[acc], acc_ph, s.abort_flag, &g_small_chain_status, kStatusEpilogueTimeout))
      return false;
    __syncwarp();
    tc_fence_after();
    return true;
  }

  __device__ void release_acc() {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&s.tempty[acc]);
    acc ^= 1;
    if (acc == 0) acc_ph ^= 1u;
  }

  // Barrier over the eight epilogue warps (bounded, unlike a named barrier).
  __device__ bool epi_barrier() {
    __syncwarp();
    if (lane == 0) mbar_arrive(s.ebar);
    const bool ok = mbar_wait_bounded(s.ebar, e_ph, s.abort_flag, &g_small_chain_status, kStatusEpilogueTimeout);
    e_ph ^= 1u;
    __syncwarp();
    return ok;
  }

  __device__ uint32_t tmem_addr(int c0) const {
    return tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc) * kAccCols +
           static_cast<uint32_t>(c0);
  }

  __device__ bool gram(int) { return sym(kNone, kNone, kNone, 1.0f, 0.0f, kMatG, kNone, 0.0f); }

  // D = alpha acc + beta C (C, D, D2 shared-memory matrices); D2 = D + gamma2 I.
  // Only the 32 x 32 blocks on or above the block diagonal are computed: each is
  // stored by rows and, transposed, into its mirror block below the diagonal
  // (a diagonal block mirrors its strict upper triangle onto its lower one), so
  // the stored matrices are exactly symmetric.
  __device__ bool sym(int, int, int C, float alpha, float beta, int D, int D2, float gamma2) {
    if (!wait_acc()) return false;
    const uint32_t r = static_cast<uint32_t>(quarter * 32 + lane);
    uint8_t* dm = s.mats + D * kMatBytes;
    uint8_t* d2m = D2 >= 0 ? s.mats + D2 * kMatBytes : nullptr;
    // This warp's blocks: row block `quarter`, column blocks 2 half and 2 half + 1.
    // Blocks below the diagonal are the mirrors of blocks (cb, quarter), which
    // their warps store.
#pragma unroll 1
    for (int q = 0; q < 2; ++q) {
      const int cb = 2 * half + q;
      if (cb < quarter) continue;
      const uint32_t c0 = static_cast<uint32_t>(cb * 32);
      float v[32];
      tmem_load_32cols(tmem_addr(static_cast<int>(c0)), v);
      uint32_t w[16];
      if (C >= 0) {
        const uint8_t* cm = s.mats + C * kMatBytes;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 u = *reinterpret_cast<const uint4*>(cm + mat_off(r, c0 + 8u * j));
          const uint32_t cw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 cf = __half22float2(*reinterpret_cast<const __half2*>(&cw[e]));
            const int k = 8 * j + 2 * e;
            w[k >> 1] = pack_half2(fmaf(beta, cf.x, alpha * v[k]), fmaf(beta, cf.y, alpha * v[k + 1]));
          }
        }
      } else {
#pragma unroll
        for (int k = 0; k < 32; k += 2) w[k >> 1] = pack_half2(alpha * v[k], alpha * v[k + 1]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(dm + mat_off(r, c0 + 8u * j)) =
            make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
      const bool diag = cb == quarter;
      uint32_t w2[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) w2[i] = w[i];
      if (d2m) {
        if (diag && static_cast<int>(r) < p.m) {
          // gamma2 on the diagonal element (column r), added to the rounded value.
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if ((static_cast<uint32_t>(lane) >> 1) != static_cast<uint32_t>(i)) continue;
            const uint32_t sh = (lane & 1) ? 16u : 0u;
            const __half h = __ushort_as_half(static_cast<unsigned short>(w2[i] >> sh));
            const uint32_t nh = __half_as_ushort(__float2half_rn(__half2float(h) + gamma2));
            w2[i] = (w2[i] & ~(0xffffu << sh)) | (nh << sh);
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(d2m + mat_off(r, c0 + 8u * j)) =
              make_uint4(w2[4 * j], w2[4 * j + 1], w2[4 * j + 2], w2[4 * j + 3]);
      }
      // Mirror: element (r, c0 + j) also goes to (c0 + j, r), as 32-bit words
      // (two adjacent columns) assembled from lane pairs: per pair of rows
      // (j, j + 1) the even lane stores row j and the odd lane row j + 1, each
      // with one value received from its partner. In a diagonal block only words
      // strictly below the diagonal, or ending on it, are stored, after the row
      // stores above have landed. A word ends on the diagonal only in an odd
      // lane's own element; its D2 copy takes that element from w2 (gamma2 added).
      __syncwarp();
      const bool odd = (lane & 1) != 0;
      const uint32_t col = r & ~1u;  // first column of this lane pair's word
      const int col_l = lane & ~1;
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const uint32_t hj = w[j >> 1] & 0xffffu, hj1 = w[j >> 1] >> 16;
        const uint32_t got = __shfl_xor_sync(0xffffffffu, odd ? hj : hj1, 1);
        const int jj = odd ? j + 1 : j;
        const uint32_t word = odd ? (got | (hj1 << 16)) : (hj | (got << 16));
        if (diag && jj <= col_l) continue;
        const uint32_t off = mat_off(c0 + static_cast<uint32_t>(jj), col);
        *reinterpret_cast<uint32_t*>(dm + off) = word;
        if (d2m) *reinterpret_cast<uint32_t*>(d2m + off) = odd ? (got | (w2[j >> 1] & 0xffff0000u)) : word;
      }
    }
    release_acc();
    fence_proxy_async_smem();  // the MMAs (async proxy) read these matrices next
    if (!epi_barrier()) return false;
    if (lane == 0) mbar_arrive(s.opnd);
    return true;
  }

  // Row `row`, columns [c0, c0 + 32) of the output (values already rounded to
  // fp16), converted to the output type.
  __device__ void write_out(int row, int c0, int ncols, const float (&v)[32]) const {
    const bool whole = c0 + 32 <= ncols;
    const int64_t base = static_cast<int64_t>(b) * p.out_bstride + static_cast<int64_t>(row) * p.out_rstride + c0;
    if (whole && p.out_vec && p.out_dtype == kF32) {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + base);
#pragma unroll
      for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else if (whole && p.out_vec) {
      uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + base);
      uint32_t w[16];
#pragma unroll
      for (int k = 0; k < 32; k += 2) {
        if (p.out_dtype == kBF16) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(v[k], v[k + 1]);
          w[k >> 1] = *reinterpret_cast<const uint32_t*>(&h);
        } else {
          w[k >> 1] = pack_half2(v[k], v[k + 1]);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k)
        if (c0 + k < ncols) store_from_float(p.out, base + k, p.out_dtype, v[k]);
    }
  }

  // Square chain: G = X X^T, a symmetric product without C.
  bool x_from_tma = false;
  uint32_t xl_ph = 0;
  __device__ bool square_gram(bool first) {
    x_from_tma = x_from_tma || first;
    return sym(kNone, kNone, kNone, 1.0f, 0.0f, kMatG, kNone, 0.0f);
  }

  // Square chain: X <- fp16(P X + a X), in place (the MMAs have read X), or, at
  // the last iteration, the output. Every block is computed (no symmetry).
  __device__ bool square_xprod(float a, bool last) {
    if (!wait_acc()) return false;
    if (x_from_tma) {
      // This product reads X as it came from the TMA load: acquire that load's
      // completion here too, not only through the MMA thread.
      if (!mbar_wait_bounded(s.xload, xl_ph, s.abort_flag, &g_small_chain_status, kStatusEpilogueTimeout))
        return false;
      xl_ph ^= 1u;
      x_from_tma = false;
    }
    const uint32_t r = static_cast<uint32_t>(quarter * 32 + lane);
    uint8_t* xm = s.mats + kMatX * kMatBytes;
#pragma unroll 1
    for (int q = 0; q < 2; ++q) {
      const uint32_t c0 = static_cast<uint32_t>((2 * half + q) * 32);
      float v[32];
      __syncwarp();
      tmem_load_32cols(tmem_addr(static_cast<int>(c0)), v);
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 u = *reinterpret_cast<const uint4*>(xm + mat_off(r, c0 + 8u * j));
        const uint32_t cw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 cf = __half22float2(*reinterpret_cast<const __half2*>(&cw[e]));
          const int k = 8 * j + 2 * e;
          w[k >> 1] = pack_half2(fmaf(a, cf.x, v[k]), fmaf(a, cf.y, v[k + 1]));
        }
      }
      if (!last) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(xm + mat_off(r, c0 + 8u * j)) =
              make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
      } else if (static_cast<int>(r) < p.m && static_cast<int>(c0) < p.m) {
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k >> 1]));
          v[k] = f.x;
          v[k + 1] = f.y;
        }
        write_out(static_cast<int>(r), static_cast<int>(c0), p.m, v);
      }
    }
    release_acc();
    if (last) {
      // Every read of this matrix's X is done: the producer may load the next one.
      __syncwarp();
      if (lane == 0) mbar_arrive(s.xready);
      return true;
    }
    fence_proxy_async_smem();
    if (!epi_barrier()) return false;
    if (lane == 0) mbar_arrive(s.opnd);
    return true;
  }

  // X-product tiles to global memory: the reset X (fp16) or the output.
  __device__ bool xprod(int xi, bool reset) {
    const int tiles = (p.n + 127) / 128;
    const int nrows = TALL ? p.n : p.m, ncols = TALL ? p.m : p.n;
    for (int t = 0; t < tiles; ++t) {
      if (!wait_acc()) return false;
      const int row = (TALL ? t * 128 : 0) + quarter * 32 + lane;
#pragma unroll 1
      for (int q = 0; q < 2; ++q) {
        const int c0 = (TALL ? 0 : t * 128) + (2 * half + q) * 32;
        float v[32];
        __syncwarp();
        tmem_load_32cols(tmem_addr((2 * half + q) * 32), v);
        if (row >= nrows || c0 >= ncols) continue;
        const bool whole = c0 + 32 <= ncols;
        if (reset) {
          __half* dst = p.x[xi ^ 1] + static_cast<int64_t>(b) * p.xb + static_cast<int64_t>(row) * p.ldx + c0;
          if (whole && p.x_vec) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              reinterpret_cast<uint4*>(dst)[j] =
                  make_uint4(pack_half2(v[8 * j], v[8 * j + 1]), pack_half2(v[8 * j + 2], v[8 * j + 3]),
                             pack_half2(v[8 * j + 4], v[8 * j + 5]), pack_half2(v[8 * j + 6], v[8 * j + 7]));
          } else {
#pragma unroll
            for (int k = 0; k < 32; ++k)
              if (c0 + k < ncols) dst[k] = __float2half_rn(v[k]);
          }
        } else {
          // The final product is rounded through fp16, then to the output type.
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = __half2float(__float2half_rn(v[k]));
          write_out(row, c0, ncols, v);
        }
      }
      release_acc();
    }
    if (reset) {
      // The producer's next TMA loads (async proxy) read what was just stored.
      fence_proxy_async_global();
      __syncwarp();
      if (lane == 0) mbar_arrive(s.xready);
    }
    return true;
  }
};

template <int MODE>
__global__ void __launch_bounds__(kThreadsSC, 1)
    small_gram_chain_kernel(const __grid_constant__ CUtensorMap map0, const __grid_constant__ CUtensorMap map1,
                            const __grid_constant__ SmallChainParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Shared s;
  s.slots = smem;
  s.mats = smem + kSlots * kSlotBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(s.mats + kMats * kMatBytes);
  s.full = bars;
  s.empty = bars + kSlots;
  s.tfull = bars + 2 * kSlots;
  s.tempty = bars + 2 * kSlots + 2;
  s.opnd = bars + 2 * kSlots + 4;
  s.xready = bars + 2 * kSlots + 5;
  s.ebar = bars + 2 * kSlots + 6;
  s.xload = bars + 2 * kSlots + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBarCount);
  s.abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], kEpiWarpsSC);
    }
    mbar_init(s.opnd, kEpiWarpsSC);
    mbar_init(s.xready, kEpiWarpsSC);
    mbar_init(s.ebar, kEpiWarpsSC);
    mbar_init(s.xload, 1);
    *s.abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map0);
    tma_prefetch_desc(&map1);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemColsSC);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait_predecessor();  // the normalised X comes from the previous kernel

  constexpr bool TALL = MODE == kTall;
  auto walk = [&](auto& role) {
    if constexpr (MODE == kSquare)
      return walk_standard(p, role);
    else
      return walk_chain(p, role);
  };
  if (warp == 0) {
    if (lane == 0) {
      ProducerRole<TALL> role(p, s, &map0, &map1);
      for (int b = blockIdx.x; b < p.batch; b += gridDim.x) {
        role.b = b;
        if (!walk(role)) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      MmaRole<TALL> role(p, s, tmem_base);
      for (int b = blockIdx.x; b < p.batch; b += gridDim.x)
        if (!walk(role)) break;
    }
  } else {
    EpilogueRole<TALL> role(p, s, tmem_base, warp, lane);
    for (int b = blockIdx.x; b < p.batch; b += gridDim.x) {
      role.b = b;
      if (!walk(role)) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*s.abort_flag) settle_for_ns(2000000ull);
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, kTmemColsSC);
  }
}

std::atomic<int> g_small_chain_enabled{1};
std::mutex g_sc_mutex;
uint32_t g_sc_attr_done[64] = {};

}  // namespace

bool small_chain_applies(int64_t batch, int64_t rows, int64_t cols) {
  if (g_small_chain_enabled.load(std::memory_order_relaxed) == 0) return false;
  const int64_t m = rows < cols ? rows : cols, n = rows < cols ? cols : rows;
  return rows != cols && m >= 1 && m <= kSmallM && n <= kSmallMaxN && batch >= 1 && batch <= (int64_t{1} << 30);
}

int small_chain_status(int* status, int clear) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_small_chain_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "read small-chain status");
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_small_chain_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "clear small-chain status");
  }
  return GNS_OK;
}

namespace {

// Fills the parameters shared by both chains and launches `MODE`.
int launch_small(int mode, int64_t batch, int64_t rows, int64_t cols, __half* x0, __half* x1, int64_t ldx, int64_t xb,
                 void* out, int out_dtype, int64_t out_bstride, int64_t out_rstride, const double* coeffs, int n_iters,
                 uint32_t reset_mask, cudaStream_t stream) {
  if (n_iters < 1 || n_iters > kMaxItersSC) return fail(GNS_ERR_ARGUMENT, "n_iters must be in [1, 32]");
  const bool tall = rows > cols;
  SmallChainParams p{};
  p.batch = static_cast<int>(batch);
  p.m = static_cast<int>(tall ? cols : rows);
  p.n = static_cast<int>(tall ? rows : cols);
  p.n_iters = n_iters;
  p.reset_mask = reset_mask;
  for (int i = 0; i < n_iters; ++i)
    for (int k = 0; k < 3; ++k) p.coef[i][k] = static_cast<float>(coeffs[3 * i + k]);
  p.x[0] = x0;
  p.x[1] = x1;
  p.ldx = ldx;
  p.xb = xb;
  p.out = out;
  p.out_dtype = out_dtype;
  p.out_bstride = out_bstride;
  p.out_rstride = out_rstride;
  const int es = dtype_size(out_dtype);
  p.out_vec = (reinterpret_cast<uintptr_t>(out) % 16 == 0 && (out_rstride * es) % 16 == 0 &&
               (batch == 1 || (out_bstride * es) % 16 == 0))
                  ? 1
                  : 0;
  p.x_vec = ((ldx * 2) % 16 == 0 && (xb * 2) % 16 == 0) ? 1 : 0;

  CUtensorMap maps[2];
  for (int i = 0; i < 2; ++i) {
    const int rc = encode_f16_tiles(&maps[i], i == 0 || x1 == nullptr ? x0 : x1, cols, rows, batch, ldx, xb, 64);
    if (rc != GNS_OK) return rc;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(GNS_ERR_DEVICE, "device index out of range");
  auto kern = mode == kSquare ? small_gram_chain_kernel<kSquare>
                              : (mode == kTall ? small_gram_chain_kernel<kTall> : small_gram_chain_kernel<kWide>);
  {
    std::lock_guard<std::mutex> lock(g_sc_mutex);
    const uint32_t bit = 1u << mode;
    if (!(g_sc_attr_done[dev] & bit)) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytesSC));
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(small chain smem)");
      g_sc_attr_done[dev] |= bit;
    }
  }
  const int sms = device_sm_count();
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(static_cast<unsigned>(batch < sms ? batch : sms), 1, 1);
  cfg.blockDim = dim3(kThreadsSC, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytesSC;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], p);
  if (e != cudaSuccess) return cuda_fail(e, "small chain kernel launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "small chain kernel launch");
  return GNS_OK;
}

}  // namespace

int launch_small_gram_chain(int64_t batch, int64_t rows, int64_t cols, __half* x0, __half* x1, int64_t ldx,
                            int64_t xb, void* out, int out_dtype, int64_t out_bstride, int64_t out_rstride,
                            const double* coeffs, int n_iters, uint32_t reset_mask, cudaStream_t stream) {
  return launch_small(rows > cols ? kTall : kWide, batch, rows, cols, x0, x1, ldx, xb, out, out_dtype, out_bstride,
                      out_rstride, coeffs, n_iters, reset_mask, stream);
}

bool small_square_applies(int64_t batch, int64_t rows, int64_t cols) {
  if (g_small_chain_enabled.load(std::memory_order_relaxed) == 0) return false;
  return rows == cols && rows >= 1 && rows <= kSmallM && batch >= 1 && batch <= (int64_t{1} << 30);
}

int launch_small_standard_chain(int64_t batch, int64_t m, __half* x0, int64_t ldx, int64_t xb, void* out,
                                int out_dtype, int64_t out_bstride, int64_t out_rstride, const double* coeffs,
                                int n_iters, cudaStream_t stream) {
  return launch_small(kSquare, batch, m, m, x0, nullptr, ldx, xb, out, out_dtype, out_bstride, out_rstride, coeffs,
                      n_iters, 0u, stream);
}

}  // namespace gns

extern "C" int gns_set_small_chain(int enabled) {
  return gns::g_small_chain_enabled.exchange(enabled ? 1 : 0);
}
