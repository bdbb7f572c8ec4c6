// HBM-bound optimizer-state kernels: Muon momentum / update and Dion3 row
// selection, NorMuon normalisation and scatter update.
//
// All kernels stream 16-byte vectors when the tensors allow it, reduce with
// warp shuffles, and round to the storage dtype at exactly the points where the
// reference's torch / CUDA code rounds.
#include <algorithm>
#include <string>

#include "../../include/gns_b200.h"
#include "gns_common.cuh"
#include "gns_host.h"

namespace gns {
namespace {

// ------------------------------------------------------------ vector I/O
template <int N>
struct Vec {
  float v[N];
};

// Loads 8 consecutive elements (idx multiple of 8, base 16-byte aligned).
__device__ __forceinline__ void ld8(const void* base, int64_t idx, int dt, float (&f)[8]) {
  if (dt == kF32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
    const float4 a = p[0], b = p[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    return;
  }
  const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + idx);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    uint32_t x = w[e];
    float2 t = (dt == kBF16) ? __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&x))
                             : __half22float2(*reinterpret_cast<__half2*>(&x));
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

__device__ __forceinline__ void st8(void* base, int64_t idx, int dt, const float (&f)[8]) {
  if (dt == kF32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(base) + idx);
    p[0] = make_float4(f[0], f[1], f[2], f[3]);
    p[1] = make_float4(f[4], f[5], f[6], f[7]);
    return;
  }
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if (dt == kBF16) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
      w[e] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __half2 h = __floats2half2_rn(f[2 * e], f[2 * e + 1]);
      w[e] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  *reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + idx) = make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__host__ __device__ inline bool al16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// ------------------------------------------------------------ Muon (K5)
constexpr int kMT = 48;           // tensors per multi-tensor launch
constexpr int kMTChunk = 32768;   // elements per CTA (8192 moved 3-6% less on B200)
constexpr int kMTThreads = 256;

struct MTArgs {
  const void* a[kMT];  // grads (momentum) / updates (apply)
  void* b[kMT];        // momenta (momentum) / params (apply)
  void* c[kMT];        // nesterov outputs (momentum)
  int64_t numel[kMT];
  float scal[kMT];     // per-tensor lr_adj (apply)
  int block_start[kMT + 1];
  int count;
};

__device__ __forceinline__ int find_tensor(const MTArgs& a, int blk) {
  int t = 0;
  while (t + 1 < a.count && a.block_start[t + 1] <= blk) ++t;
  return t;
}

// m <- round_m(round_m(g) + mu * m); u <- round_u(g + mu * m_new)
// G, M, U >= 0 fix the dtypes at compile time, so the unrolled vector loop has
// no dtype branches and keeps several iterations' loads in flight (on B200 the
// bf16 instantiation moves 6.8 TB/s on Llama-3-8B shapes against 4.5 TB/s with
// the dtypes read from the arguments). -1 takes them from the arguments: the
// fallback for rare combinations.
template <int G, int M, int U>
__global__ void __launch_bounds__(kMTThreads) muon_momentum_kernel(const MTArgs args, int g_rt, int m_rt, int u_rt,
                                                                   float mu, int nesterov) {
  const int g_dt = G >= 0 ? G : g_rt;
  const int m_dt = M >= 0 ? M : m_rt;
  const int u_dt = U >= 0 ? U : u_rt;
  const int t = find_tensor(args, blockIdx.x);
  const int64_t n = args.numel[t];
  const int64_t start = static_cast<int64_t>(blockIdx.x - args.block_start[t]) * kMTChunk;
  const int64_t end = min(n, start + kMTChunk);
  const void* g = args.a[t];
  void* m = args.b[t];
  void* u = args.c[t];
  // A tensor without an update output (u == nullptr) only advances its momentum.
  const bool write_u = nesterov && u != nullptr;
  const bool vec = al16(g) && al16(m) && (!write_u || al16(u));
  if (vec) {
    const int64_t vend = start + ((end - start) / 8) * 8;
#pragma unroll 4
    for (int64_t i = start + threadIdx.x * 8; i < vend; i += kMTThreads * 8) {
      float gf[8], mf[8], uf[8];
      ld8(g, i, g_dt, gf);
      ld8(m, i, m_dt, mf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float gm = round_to(gf[e], m_dt);
        mf[e] = (mu == 0.0f) ? gm : round_to(fmaf(mu, mf[e], gm), m_dt);
        uf[e] = fmaf(mu, mf[e], gf[e]);
      }
      st8(m, i, m_dt, mf);
      if (write_u) st8(u, i, u_dt, uf);
    }
    for (int64_t i = vend + threadIdx.x; i < end; i += kMTThreads) {
      const float gf = load_as_float(g, i, g_dt);
      const float gm = round_to(gf, m_dt);
      const float mf = (mu == 0.0f) ? gm : round_to(fmaf(mu, load_as_float(m, i, m_dt), gm), m_dt);
      store_from_float(m, i, m_dt, mf);
      if (write_u) store_from_float(u, i, u_dt, fmaf(mu, mf, gf));
    }
  } else {
    for (int64_t i = start + threadIdx.x; i < end; i += kMTThreads) {
      const float gf = load_as_float(g, i, g_dt);
      const float gm = round_to(gf, m_dt);
      const float mf = (mu == 0.0f) ? gm : round_to(fmaf(mu, load_as_float(m, i, m_dt), gm), m_dt);
      store_from_float(m, i, m_dt, mf);
      if (write_u) store_from_float(u, i, u_dt, fmaf(mu, mf, gf));
    }
  }
}

// p <- round(p * decay) (optional); p <- round(p - lr_adj * o)
// P, O >= 0 fix the dtypes at compile time (as in muon_momentum_kernel).
template <int P, int O>
__global__ void __launch_bounds__(kMTThreads) muon_apply_kernel(const MTArgs args, int p_rt, int o_rt, float decay,
                                                                int apply_decay) {
  const int p_dt = P >= 0 ? P : p_rt;
  const int o_dt = O >= 0 ? O : o_rt;
  const int t = find_tensor(args, blockIdx.x);
  const int64_t n = args.numel[t];
  const int64_t start = static_cast<int64_t>(blockIdx.x - args.block_start[t]) * kMTChunk;
  const int64_t end = min(n, start + kMTChunk);
  const void* o = args.a[t];
  void* p = args.b[t];
  const float nlr = -args.scal[t];
  const bool vec = al16(o) && al16(p);
  if (vec) {
    const int64_t vend = start + ((end - start) / 8) * 8;
#pragma unroll 4
    for (int64_t i = start + threadIdx.x * 8; i < vend; i += kMTThreads * 8) {
      float pf[8], of[8];
      ld8(p, i, p_dt, pf);
      ld8(o, i, o_dt, of);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float x = apply_decay ? round_to(pf[e] * decay, p_dt) : pf[e];
        pf[e] = fmaf(nlr, of[e], x);
      }
      st8(p, i, p_dt, pf);
    }
    for (int64_t i = vend + threadIdx.x; i < end; i += kMTThreads) {
      float x = load_as_float(p, i, p_dt);
      if (apply_decay) x = round_to(x * decay, p_dt);
      store_from_float(p, i, p_dt, fmaf(nlr, load_as_float(o, i, o_dt), x));
    }
  } else {
    for (int64_t i = start + threadIdx.x; i < end; i += kMTThreads) {
      float x = load_as_float(p, i, p_dt);
      if (apply_decay) x = round_to(x * decay, p_dt);
      store_from_float(p, i, p_dt, fmaf(nlr, load_as_float(o, i, o_dt), x));
    }
  }
}

// The dtype combinations Muon meets (same-dtype state; bf16 or fp16 gradients
// with fp32 momentum) get their own instantiation; the others run the
// runtime-dtype kernel.
void launch_muon_momentum(int blocks, cudaStream_t st, const MTArgs& a, int g, int m, int u, float mu, int nesterov) {
  const dim3 grid(static_cast<unsigned>(blocks));
  if (g == kBF16 && m == kBF16 && u == kBF16)
    muon_momentum_kernel<kBF16, kBF16, kBF16><<<grid, kMTThreads, 0, st>>>(a, g, m, u, mu, nesterov);
  else if (g == kF32 && m == kF32 && u == kF32)
    muon_momentum_kernel<kF32, kF32, kF32><<<grid, kMTThreads, 0, st>>>(a, g, m, u, mu, nesterov);
  else if (g == kF16 && m == kF16 && u == kF16)
    muon_momentum_kernel<kF16, kF16, kF16><<<grid, kMTThreads, 0, st>>>(a, g, m, u, mu, nesterov);
  else if (g == kBF16 && m == kF32 && u == kF32)
    muon_momentum_kernel<kBF16, kF32, kF32><<<grid, kMTThreads, 0, st>>>(a, g, m, u, mu, nesterov);
  else if (g == kF16 && m == kF32 && u == kF32)
    muon_momentum_kernel<kF16, kF32, kF32><<<grid, kMTThreads, 0, st>>>(a, g, m, u, mu, nesterov);
  else
    muon_momentum_kernel<-1, -1, -1><<<grid, kMTThreads, 0, st>>>(a, g, m, u, mu, nesterov);
}

void launch_muon_apply(int blocks, cudaStream_t st, const MTArgs& a, int p, int o, float decay, int apply_decay) {
  const dim3 grid(static_cast<unsigned>(blocks));
  if (p == kBF16 && o == kBF16)
    muon_apply_kernel<kBF16, kBF16><<<grid, kMTThreads, 0, st>>>(a, p, o, decay, apply_decay);
  else if (p == kF32 && o == kF32)
    muon_apply_kernel<kF32, kF32><<<grid, kMTThreads, 0, st>>>(a, p, o, decay, apply_decay);
  else if (p == kF16 && o == kF16)
    muon_apply_kernel<kF16, kF16><<<grid, kMTThreads, 0, st>>>(a, p, o, decay, apply_decay);
  else
    muon_apply_kernel<-1, -1><<<grid, kMTThreads, 0, st>>>(a, p, o, decay, apply_decay);
}

// ------------------------------------------------------------ Dion3 (K6)
constexpr int kRowThreads = 256;  // 8 warps, one row per warp

// Where each matrix of a Dion3 launch lives: count == 0 means one contiguous
// stack (matrix b at base[0] + b * stride bytes); otherwise base[b] holds matrix
// b of a list of separate same-shape tensors (at most kD3 per launch).
constexpr int kD3 = 64;
struct MatPtrs {
  void* base[kD3];
  int count;
};

__device__ __forceinline__ char* mat_at(const MatPtrs& t, int64_t b, int64_t stride_bytes) {
  return t.count ? static_cast<char*>(t.base[b]) : static_cast<char*>(t.base[0]) + b * stride_bytes;
}

// m <- round(m + g); p <- round(p * pdecay) if pdecay != 1; norms[row] = sum |m|
// (row counts over the launch's matrices, `rows` per matrix).
__global__ void __launch_bounds__(kRowThreads) dion3_momentum_rownorm_kernel(const MatPtrs mt, const MatPtrs gt,
                                                                             const MatPtrs pt, int dt, int64_t rows,
                                                                             int64_t nrows, int64_t cols,
                                                                             float pdecay, int vec,
                                                                             float* __restrict__ norms) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kRowThreads / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= nrows) return;
  const int64_t b = row / rows;
  const int64_t stride = rows * cols * dtype_size(dt);
  void* m = mat_at(mt, b, stride);
  const void* g = mat_at(gt, b, stride);
  const bool decay = pdecay != 1.0f;
  void* p = decay ? mat_at(pt, b, stride) : nullptr;
  const int64_t base = (row - b * rows) * cols;
  float acc = 0.0f;
  if (vec) {
    for (int64_t c = lane * 8; c < cols; c += 32 * 8) {
      float mf[8], gf[8];
      ld8(m, base + c, dt, mf);
      ld8(g, base + c, dt, gf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        mf[e] = round_to(mf[e] + gf[e], dt);
        acc += fabsf(mf[e]);
      }
      st8(m, base + c, dt, mf);
      if (decay) {
        float pf[8];
        ld8(p, base + c, dt, pf);
#pragma unroll
        for (int e = 0; e < 8; ++e) pf[e] = pf[e] * pdecay;
        st8(p, base + c, dt, pf);
      }
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) {
      const float mf = round_to(load_as_float(m, base + c, dt) + load_as_float(g, base + c, dt), dt);
      store_from_float(m, base + c, dt, mf);
      acc += fabsf(mf);
      if (decay) store_from_float(p, base + c, dt, load_as_float(p, base + c, dt) * pdecay);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) norms[row] = acc;
}

// ------------------------------------------------------------ Dion3 (K7)
constexpr int kSelThreads = 1024;

__device__ __forceinline__ uint32_t norm_key(float x) {
  // Row L1 norms are >= 0 (or NaN), so the raw bit pattern orders them; NaN sorts highest.
  return __float_as_uint(x) & 0x7fffffffu;
}

// Block-wide exclusive scan of one int per thread; returns the exclusive prefix, *total = sum.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int w = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) warp_tot[lane] = w;  // inclusive
  }
  __syncthreads();
  const int before = (warp > 0 ? warp_tot[warp - 1] : 0) + x - v;
  if (total) *total = warp_tot[(blockDim.x >> 5) - 1];
  __syncthreads();
  return before;
}

// One CTA per matrix: radix-select the k-th largest row norm, then emit the
// indices of the k largest rows in ascending order (ties at the threshold are
// taken lowest index first).
__global__ void __launch_bounds__(kSelThreads) dion3_topk_kernel(const float* __restrict__ norms, int64_t rows,
                                                                 int64_t k, int64_t* __restrict__ indices) {
  __shared__ int hist[256];
  __shared__ int warp_tot[32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_need;
  const float* nb = norms + static_cast<int64_t>(blockIdx.x) * rows;
  int64_t* out = indices + static_cast<int64_t>(blockIdx.x) * k;

  uint32_t prefix = 0, mask = 0;
  int need = static_cast<int>(k);
  const int lane = threadIdx.x & 31;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    // Lanes of a warp that fall into the same bin add their count with one
    // atomic (row norms cluster in a few exponent bins, so per-row atomics on
    // one shared word serialised).
    for (int64_t base = 0; base < rows; base += blockDim.x) {
      const int64_t r = base + threadIdx.x;
      int bin = 256;
      if (r < rows) {
        const uint32_t key = norm_key(nb[r]);
        if ((key & mask) == prefix) bin = static_cast<int>((key >> shift) & 0xffu);
      }
      const unsigned peers = __match_any_sync(0xffffffffu, bin);
      if (bin < 256 && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
    }
    __syncthreads();
    // Digit = the bin d holding the need-th largest key: with above(d) the count
    // in bins above d, above(d) < need <= above(d) + hist[d]. Thread t scans bin
    // 255 - t, so its exclusive prefix is above(255 - t).
    const int d = 255 - static_cast<int>(threadIdx.x);
    const int h = threadIdx.x < 256 ? hist[d] : 0;
    const int above = block_exclusive_scan(h, warp_tot, nullptr);
    if (threadIdx.x < 256 && above < need && above + h >= need) {
      s_prefix = prefix | (static_cast<uint32_t>(d) << shift);
      s_need = need - above;
    }
    __syncthreads();
    prefix = s_prefix;
    need = s_need;
    mask |= 0xffu << shift;
    __syncthreads();
  }
  const uint32_t thr = prefix;  // key of the k-th largest; `need` ties at thr are taken

  // Each thread owns a contiguous run of rows so that scans preserve index order.
  const int64_t per = (rows + blockDim.x - 1) / blockDim.x;
  const int64_t r0 = min(rows, static_cast<int64_t>(threadIdx.x) * per);
  const int64_t r1 = min(rows, r0 + per);
  int eq = 0;
  for (int64_t r = r0; r < r1; ++r) eq += (norm_key(nb[r]) == thr);
  const int eq_before = block_exclusive_scan(eq, warp_tot, nullptr);
  int take = 0;
  {
    int e = eq_before;
    for (int64_t r = r0; r < r1; ++r) {
      const uint32_t key = norm_key(nb[r]);
      if (key > thr) {
        ++take;
      } else if (key == thr) {
        if (e < need) ++take;
        ++e;
      }
    }
  }
  const int pos0 = block_exclusive_scan(take, warp_tot, nullptr);
  int pos = pos0;
  int e = eq_before;
  for (int64_t r = r0; r < r1; ++r) {
    const uint32_t key = norm_key(nb[r]);
    bool sel = key > thr;
    if (key == thr) {
      sel = e < need;
      ++e;
    }
    if (sel) out[pos++] = r;
  }
}

__global__ void iota_kernel(int64_t* __restrict__ indices, int64_t batch, int64_t rows) {
  const int64_t n = batch * rows;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    indices[i] = i % rows;
}

// sel[b, s, :] = bf16(m[b, idx, :]); m[b, idx, :] = round(m * decay). One warp per selected row.
__global__ void __launch_bounds__(kRowThreads) dion3_gather_decay_kernel(const MatPtrs mt, int dt, int64_t rows,
                                                                         int64_t cols, int64_t k, int64_t nsel,
                                                                         const int64_t* __restrict__ indices,
                                                                         float decay, int vec,
                                                                         __nv_bfloat16* __restrict__ sel) {
  const int64_t srow = static_cast<int64_t>(blockIdx.x) * (kRowThreads / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (srow >= nsel) return;
  const int64_t b = srow / k;
  const int64_t r = indices[srow];
  if (r < 0 || r >= rows) return;
  void* m = mat_at(mt, b, rows * cols * dtype_size(dt));
  const int64_t mbase = r * cols;
  const int64_t sbase = srow * cols;
  if (vec) {
#pragma unroll 4
    for (int64_t c = lane * 8; c < cols; c += 32 * 8) {
      float f[8];
      ld8(m, mbase + c, dt, f);
      st8(sel, sbase + c, kBF16, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] *= decay;
      st8(m, mbase + c, dt, f);
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) {
      const float f = load_as_float(m, mbase + c, dt);
      sel[sbase + c] = __float2bfloat16_rn(f);
      store_from_float(m, mbase + c, dt, f * decay);
    }
  }
}

// ------------------------------------------------------------ Dion3 (K8)
// Per selected row: ss_u = sum u^2; v <- beta2 v + (1 - beta2) ss_u / cols;
// denom = sqrt(v) + eps; ss_n = sum (u / denom)^2.
__global__ void __launch_bounds__(kRowThreads) dion3_rowstats_kernel(const void* u, int u_dt, int64_t u_bstride,
                                                                     int64_t u_rstride, int64_t rows, int64_t cols,
                                                                     int64_t k, int64_t nsel,
                                                                     const int64_t* __restrict__ indices,
                                                                     const MatPtrs vt, float beta2,
                                                                     float eps, int vec, float* __restrict__ stats) {
  const int64_t srow = static_cast<int64_t>(blockIdx.x) * (kRowThreads / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (srow >= nsel) return;
  const int64_t b = srow / k, s = srow % k;
  const int64_t r = indices[srow];
  const int64_t ubase = b * u_bstride + s * u_rstride;
  float ss = 0.0f;
  if (vec) {
#pragma unroll 4
    for (int64_t c = lane * 8; c < cols; c += 32 * 8) {
      float f[8];
      ld8(u, ubase + c, u_dt, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) {
      const float f = load_as_float(u, ubase + c, u_dt);
      ss = fmaf(f, f, ss);
    }
  }
  ss = warp_sum(ss);
  float denom = 0.0f;
  if (r >= 0 && r < rows) {
    float* variance = reinterpret_cast<float*>(mat_at(vt, b, rows * static_cast<int64_t>(sizeof(float))));
    const float v = beta2 * variance[r] + (1.0f - beta2) * (ss / static_cast<float>(cols));
    __syncwarp();
    if (lane == 0) variance[r] = v;
    denom = sqrtf(v) + eps;
  }
  float sn = 0.0f;
  if (denom > 0.0f) {
    if (vec) {
#pragma unroll 4
      for (int64_t c = lane * 8; c < cols; c += 32 * 8) {
        float f[8];
        ld8(u, ubase + c, u_dt, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float q = __fdiv_rn(f[e], denom);
          sn = fmaf(q, q, sn);
        }
      }
    } else {
      for (int64_t c = lane; c < cols; c += 32) {
        const float q = __fdiv_rn(load_as_float(u, ubase + c, u_dt), denom);
        sn = fmaf(q, q, sn);
      }
    }
  }
  sn = warp_sum(sn);
  if (lane == 0) {
    stats[3 * srow + 0] = ss;
    stats[3 * srow + 1] = sn;
    stats[3 * srow + 2] = denom;
  }
}

// One CTA per matrix: totals[b] = (sqrt(sum ss_u), max(sqrt(sum ss_n), eps)), deterministic order.
__global__ void __launch_bounds__(256) dion3_totals_kernel(const float* __restrict__ stats, int64_t k, float eps,
                                                           float* __restrict__ totals) {
  __shared__ float red_u[8], red_n[8];
  const int64_t b = blockIdx.x;
  float su = 0.0f, sn = 0.0f;
  for (int64_t s = threadIdx.x; s < k; s += blockDim.x) {
    su += stats[3 * (b * k + s) + 0];
    sn += stats[3 * (b * k + s) + 1];
  }
  su = warp_sum(su);
  sn = warp_sum(sn);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red_u[warp] = su;
    red_n[warp] = sn;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float tu = 0.0f, tn = 0.0f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
      tu += red_u[w];
      tn += red_n[w];
    }
    totals[2 * b + 0] = sqrtf(tu);
    totals[2 * b + 1] = fmaxf(sqrtf(tn), eps);
  }
}

// p <- round(p * decay) over each matrix of the launch (blockIdx.y = matrix).
__global__ void decay_kernel(const MatPtrs pt, int dt, int64_t per_matrix, float decay) {
  void* p = mat_at(pt, blockIdx.y, per_matrix * dtype_size(dt));
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < per_matrix;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    store_from_float(p, i, dt, load_as_float(p, i, dt) * decay);
}

// p[b, idx, c] = round(p + round(-lr_adj * round(n * orig / normd))), n = u / denom.
__global__ void __launch_bounds__(kRowThreads) dion3_apply_kernel(const MatPtrs pt, int p_dt, const void* u, int u_dt,
                                                                  int64_t u_bstride, int64_t u_rstride, int64_t rows,
                                                                  int64_t cols, int64_t k, int64_t nsel,
                                                                  const int64_t* __restrict__ indices,
                                                                  const float* __restrict__ stats,
                                                                  const float* __restrict__ totals, float lr_adj,
                                                                  int vec) {
  const int64_t srow = static_cast<int64_t>(blockIdx.x) * (kRowThreads / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (srow >= nsel) return;
  const int64_t b = srow / k, s = srow % k;
  const int64_t r = indices[srow];
  if (r < 0 || r >= rows) return;
  const float denom = stats[3 * srow + 2];
  const float orig = totals[2 * b + 0], normd = totals[2 * b + 1];
  const int64_t ubase = b * u_bstride + s * u_rstride;
  void* p = mat_at(pt, b, rows * cols * dtype_size(p_dt));
  const int64_t pbase = r * cols;
  if (vec) {
#pragma unroll 4
    for (int64_t c = lane * 8; c < cols; c += 32 * 8) {
      float uf[8], pf[8];
      ld8(u, ubase + c, u_dt, uf);
      ld8(p, pbase + c, p_dt, pf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float nrm = __fdiv_rn(uf[e], denom);
        const float scaled = round_to(__fdiv_rn(nrm * orig, normd), p_dt);
        const float upd = round_to(-lr_adj * scaled, p_dt);
        pf[e] = pf[e] + upd;
      }
      st8(p, pbase + c, p_dt, pf);
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) {
      const float nrm = __fdiv_rn(load_as_float(u, ubase + c, u_dt), denom);
      const float scaled = round_to(__fdiv_rn(nrm * orig, normd), p_dt);
      const float upd = round_to(-lr_adj * scaled, p_dt);
      store_from_float(p, pbase + c, p_dt, load_as_float(p, pbase + c, p_dt) + upd);
    }
  }
}

// normalized[srow] = u[srow] / denom (fp32), one warp per selected row; rows
// with an out-of-range index are left untouched.
__global__ void __launch_bounds__(kRowThreads) dion3_write_normalized_kernel(
    const void* u, int u_dt, int64_t u_bstride, int64_t u_rstride, int64_t rows, int64_t cols, int64_t k, int64_t nsel,
    const int64_t* __restrict__ indices, const float* __restrict__ stats, float* __restrict__ normalized) {
  const int64_t srow = static_cast<int64_t>(blockIdx.x) * (kRowThreads / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (srow >= nsel) return;
  const int64_t r = indices[srow];
  if (r < 0 || r >= rows) return;
  const int64_t b = srow / k, s = srow % k;
  const float denom = stats[3 * srow + 2];
  const int64_t ubase = b * u_bstride + s * u_rstride;
  for (int64_t c = lane; c < cols; c += 32)
    normalized[srow * cols + c] = __fdiv_rn(load_as_float(u, ubase + c, u_dt), denom);
}

// squared_norms[b] = (sum of the rows' |u|^2, sum of the rows' |n|^2), one CTA per
// matrix, in the summation order of dion3_totals_kernel.
__global__ void __launch_bounds__(256) dion3_sums_kernel(const float* __restrict__ stats, int64_t k,
                                                         float* __restrict__ squared_norms) {
  __shared__ float red_u[8], red_n[8];
  const int64_t b = blockIdx.x;
  float su = 0.0f, sn = 0.0f;
  for (int64_t s = threadIdx.x; s < k; s += blockDim.x) {
    su += stats[3 * (b * k + s) + 0];
    sn += stats[3 * (b * k + s) + 1];
  }
  su = warp_sum(su);
  sn = warp_sum(sn);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red_u[warp] = su;
    red_n[warp] = sn;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float tu = 0.0f, tn = 0.0f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
      tu += red_u[w];
      tn += red_n[w];
    }
    squared_norms[2 * b + 0] = tu;
    squared_norms[2 * b + 1] = tn;
  }
}

// p[b, idx, c] = round(p + round(-lr_adj * round(n * orig / normd))) for a stored
// fp32 normalized update n, orig = sqrt(sum |u|^2), normd = max(sqrt(sum |n|^2), eps).
__global__ void __launch_bounds__(kRowThreads) dion3_apply_normalized_kernel(
    const MatPtrs pt, int p_dt, const float* __restrict__ normalized, int64_t rows, int64_t cols, int64_t k, int64_t nsel,
    const int64_t* __restrict__ indices, const float* __restrict__ squared_norms, float lr_adj, float eps) {
  const int64_t srow = static_cast<int64_t>(blockIdx.x) * (kRowThreads / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (srow >= nsel) return;
  const int64_t b = srow / k;
  const int64_t r = indices[srow];
  if (r < 0 || r >= rows) return;
  const float orig = sqrtf(squared_norms[2 * b + 0]);
  const float normd = fmaxf(sqrtf(squared_norms[2 * b + 1]), eps);
  void* p = mat_at(pt, b, rows * cols * dtype_size(p_dt));
  const int64_t pbase = r * cols;
  for (int64_t c = lane; c < cols; c += 32) {
    const float scaled = round_to(__fdiv_rn(normalized[srow * cols + c] * orig, normd), p_dt);
    const float upd = round_to(-lr_adj * scaled, p_dt);
    store_from_float(p, pbase + c, p_dt, load_as_float(p, pbase + c, p_dt) + upd);
  }
}

// ------------------------------------------------------- AdamW / Lion groups
// Multi-tensor versions of the reference's per-parameter torch sequences
// (muon.py:516-583): one launch per 32 tensors instead of about ten kernels and
// a host synchronisation per parameter. Every intermediate is rounded to the
// dtype of the torch tensor that would hold it (S = state, P = parameter).
constexpr int kMT4 = 32;

struct MT4Args {
  const void* g[kMT4];  // gradients
  void* p[kMT4];        // parameters
  void* s1[kMT4];       // exp_avg (AdamW) / momentum_buffer (Lion)
  void* s2[kMT4];       // exp_avg_sq (AdamW)
  int64_t numel[kMT4];
  float lr_bc1[kMT4];   // AdamW: float(lr / (1 - beta1^step))
  float inv_bc2[kMT4];  // AdamW: float(1 / sqrt(1 - beta2^step)), the reciprocal formed in double
  int block_start[kMT4 + 1];
  int count;
};

__device__ __forceinline__ int find_tensor4(const MT4Args& a, int blk) {
  int t = 0;
  while (t + 1 < a.count && a.block_start[t + 1] <= blk) ++t;
  return t;
}

struct AdamWScalars {
  float beta1, one_minus_beta1, beta2, one_minus_beta2, epsilon, decay;
  int apply_decay;
};

// exp_avg.mul_(b1).add_(g, alpha=1-b1); exp_avg_sq.mul_(b2).addcmul_(g, g, value=1-b2);
// p.mul_(1-lr wd); denom = exp_avg_sq.sqrt().div_(sqrt(bc2)).add_(eps);
// p.sub_(exp_avg.div(denom).mul(lr/bc1)). A division by a host scalar runs as a
// multiplication by its reciprocal (formed on the host in double and rounded to
// float), as torch's CUDA division does. torch's
// `a + alpha * b` and `a + value * (b * c)` compile to one fma (after b * c);
// every other step is an explicitly rounded intrinsic so that nothing else fuses.
__device__ __forceinline__ void adamw_element(float g, float& p, float& m, float& v, int p_dt, int s_dt,
                                              const AdamWScalars& k, float lr_bc1, float inv_bc2) {
  const float gs = round_to(g, s_dt);
  m = round_to(__fmul_rn(m, k.beta1), s_dt);
  m = round_to(fmaf(k.one_minus_beta1, gs, m), s_dt);
  v = round_to(__fmul_rn(v, k.beta2), s_dt);
  v = round_to(fmaf(k.one_minus_beta2, __fmul_rn(gs, gs), v), s_dt);
  if (k.apply_decay) p = round_to(__fmul_rn(p, k.decay), p_dt);
  float d = round_to(sqrtf(v), s_dt);
  d = round_to(__fmul_rn(d, inv_bc2), s_dt);
  d = round_to(__fadd_rn(d, k.epsilon), s_dt);
  const float q = round_to(__fdiv_rn(m, d), s_dt);
  const float u = round_to(__fmul_rn(q, lr_bc1), s_dt);
  p = round_to(__fsub_rn(p, round_to(u, p_dt)), p_dt);
}

__global__ void __launch_bounds__(kMTThreads) adamw_kernel(const MT4Args args, int g_dt, int p_dt, int s_dt,
                                                           const AdamWScalars k) {
  const int t = find_tensor4(args, blockIdx.x);
  const int64_t n = args.numel[t];
  const int64_t start = static_cast<int64_t>(blockIdx.x - args.block_start[t]) * kMTChunk;
  const int64_t end = min(n, start + kMTChunk);
  const void* g = args.g[t];
  void* p = args.p[t];
  void* m = args.s1[t];
  void* v = args.s2[t];
  const float lr_bc1 = args.lr_bc1[t], inv_bc2 = args.inv_bc2[t];
  const bool vec = al16(g) && al16(p) && al16(m) && al16(v);
  int64_t i = start;
  if (vec) {
    const int64_t vend = start + ((end - start) / 8) * 8;
    for (i = start + threadIdx.x * 8; i < vend; i += kMTThreads * 8) {
      float gf[8], pf[8], mf[8], vf[8];
      ld8(g, i, g_dt, gf);
      ld8(p, i, p_dt, pf);
      ld8(m, i, s_dt, mf);
      ld8(v, i, s_dt, vf);
#pragma unroll
      for (int e = 0; e < 8; ++e) adamw_element(gf[e], pf[e], mf[e], vf[e], p_dt, s_dt, k, lr_bc1, inv_bc2);
      st8(p, i, p_dt, pf);
      st8(m, i, s_dt, mf);
      st8(v, i, s_dt, vf);
    }
    i = vend;
  }
  for (int64_t j = i + threadIdx.x; j < end; j += kMTThreads) {
    float pf = load_as_float(p, j, p_dt), mf = load_as_float(m, j, s_dt), vf = load_as_float(v, j, s_dt);
    adamw_element(load_as_float(g, j, g_dt), pf, mf, vf, p_dt, s_dt, k, lr_bc1, inv_bc2);
    store_from_float(p, j, p_dt, pf);
    store_from_float(m, j, s_dt, mf);
    store_from_float(v, j, s_dt, vf);
  }
}

struct LionScalars {
  float beta1, one_minus_beta1, beta2, one_minus_beta2, lr, decay;
  int apply_decay;
};

// d = buf.mul(b1).add(g, alpha=1-b1); p.mul_(1-lr wd); p.sub_(d.sign().mul(lr));
// buf.mul_(b2).add_(g, alpha=1-b2)
__device__ __forceinline__ void lion_element(float g, float& p, float& b, int p_dt, int s_dt, const LionScalars& k) {
  const float gs = round_to(g, s_dt);
  float d = round_to(__fmul_rn(b, k.beta1), s_dt);
  d = round_to(fmaf(k.one_minus_beta1, gs, d), s_dt);
  if (k.apply_decay) p = round_to(__fmul_rn(p, k.decay), p_dt);
  const float sg = (d > 0.0f) ? 1.0f : ((d < 0.0f) ? -1.0f : (d == 0.0f ? 0.0f : d));
  const float step = round_to(__fmul_rn(sg, k.lr), s_dt);
  p = round_to(__fsub_rn(p, round_to(step, p_dt)), p_dt);
  b = round_to(__fmul_rn(b, k.beta2), s_dt);
  b = round_to(fmaf(k.one_minus_beta2, gs, b), s_dt);
}

__global__ void __launch_bounds__(kMTThreads) lion_kernel(const MT4Args args, int g_dt, int p_dt, int s_dt,
                                                          const LionScalars k) {
  const int t = find_tensor4(args, blockIdx.x);
  const int64_t n = args.numel[t];
  const int64_t start = static_cast<int64_t>(blockIdx.x - args.block_start[t]) * kMTChunk;
  const int64_t end = min(n, start + kMTChunk);
  const void* g = args.g[t];
  void* p = args.p[t];
  void* b = args.s1[t];
  const bool vec = al16(g) && al16(p) && al16(b);
  int64_t i = start;
  if (vec) {
    const int64_t vend = start + ((end - start) / 8) * 8;
    for (i = start + threadIdx.x * 8; i < vend; i += kMTThreads * 8) {
      float gf[8], pf[8], bf[8];
      ld8(g, i, g_dt, gf);
      ld8(p, i, p_dt, pf);
      ld8(b, i, s_dt, bf);
#pragma unroll
      for (int e = 0; e < 8; ++e) lion_element(gf[e], pf[e], bf[e], p_dt, s_dt, k);
      st8(p, i, p_dt, pf);
      st8(b, i, s_dt, bf);
    }
    i = vend;
  }
  for (int64_t j = i + threadIdx.x; j < end; j += kMTThreads) {
    float pf = load_as_float(p, j, p_dt), bf = load_as_float(b, j, s_dt);
    lion_element(load_as_float(g, j, g_dt), pf, bf, p_dt, s_dt, k);
    store_from_float(p, j, p_dt, pf);
    store_from_float(b, j, s_dt, bf);
  }
}

// Fills one launch's tensor table from [off, off + kMT4); returns its block count.
int fill_mt4(MT4Args& a, int off, int count, const void* const* g, void* const* p, void* const* s1, void* const* s2,
             const int64_t* numel, const float* lr_bc1, const float* inv_bc2, int* rc) {
  int blocks = 0;
  a.count = 0;
  for (int i = off; i < count && i < off + kMT4; ++i) {
    if (numel[i] < 0) {
      *rc = fail(GNS_ERR_ARGUMENT, "negative numel");
      return 0;
    }
    const int j = a.count++;
    a.g[j] = g[i];
    a.p[j] = p[i];
    a.s1[j] = s1[i];
    a.s2[j] = s2 ? s2[i] : nullptr;
    a.numel[j] = numel[i];
    a.lr_bc1[j] = lr_bc1 ? lr_bc1[i] : 0.0f;
    a.inv_bc2[j] = inv_bc2 ? inv_bc2[i] : 0.0f;
    a.block_start[j] = blocks;
    const int64_t nb = (numel[i] + kMTChunk - 1) / kMTChunk;
    if (blocks + nb > (1ll << 30)) {
      *rc = fail(GNS_ERR_UNSUPPORTED, "tensor list too large");
      return 0;
    }
    blocks += static_cast<int>(nb);
  }
  a.block_start[a.count] = blocks;
  return blocks;
}

int blocks_for(int64_t items, int per_block) { return static_cast<int>((items + per_block - 1) / per_block); }

}  // namespace
}  // namespace gns

using namespace gns;

extern "C" {

int gns_muon_momentum(int count, const void* const* grads, void* const* moms, void* const* updates,
                      const int64_t* numel, int g_dtype, int m_dtype, int u_dtype, float mu, int nesterov,
                      gns_stream_t stream) {
  clear_error();
  if (count < 0 || (count > 0 && (grads == nullptr || moms == nullptr || numel == nullptr)))
    return fail(GNS_ERR_ARGUMENT, "bad tensor list");
  if (nesterov && count > 0 && updates == nullptr) return fail(GNS_ERR_ARGUMENT, "nesterov needs update outputs");
  for (int dt : {g_dtype, m_dtype, u_dtype})
    if (dt < 0 || dt > 2) return fail(GNS_ERR_ARGUMENT, "bad dtype");
  if (count == 0) return GNS_OK;
  int rc = check_device();
  if (rc != GNS_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  for (int off = 0; off < count; off += kMT) {
    MTArgs a{};
    int blocks = 0;
    a.count = 0;
    for (int i = off; i < count && i < off + kMT; ++i) {
      if (numel[i] < 0) return fail(GNS_ERR_ARGUMENT, "negative numel");
      const int j = a.count++;
      a.a[j] = grads[i];
      a.b[j] = moms[i];
      a.c[j] = nesterov ? updates[i] : nullptr;
      a.numel[j] = numel[i];
      a.block_start[j] = blocks;
      const int64_t nb = (numel[i] + kMTChunk - 1) / kMTChunk;
      if (blocks + nb > (1ll << 30)) return fail(GNS_ERR_UNSUPPORTED, "tensor list too large");
      blocks += static_cast<int>(nb);
    }
    a.block_start[a.count] = blocks;
    if (blocks == 0) continue;
    launch_muon_momentum(blocks, st, a, g_dtype, m_dtype, u_dtype, mu, nesterov ? 1 : 0);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "muon momentum kernel");
  return GNS_OK;
}

int gns_muon_apply(int count, void* const* params, const void* const* updates, const int64_t* numel, int p_dtype,
                   int o_dtype, float decay, int apply_decay, const float* lr_adj, gns_stream_t stream) {
  clear_error();
  if (count < 0 || (count > 0 && (params == nullptr || updates == nullptr || numel == nullptr || lr_adj == nullptr)))
    return fail(GNS_ERR_ARGUMENT, "bad tensor list");
  for (int dt : {p_dtype, o_dtype})
    if (dt < 0 || dt > 2) return fail(GNS_ERR_ARGUMENT, "bad dtype");
  if (count == 0) return GNS_OK;
  int rc = check_device();
  if (rc != GNS_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  for (int off = 0; off < count; off += kMT) {
    MTArgs a{};
    int blocks = 0;
    for (int i = off; i < count && i < off + kMT; ++i) {
      if (numel[i] < 0) return fail(GNS_ERR_ARGUMENT, "negative numel");
      const int j = a.count++;
      a.a[j] = updates[i];
      a.b[j] = params[i];
      a.numel[j] = numel[i];
      a.scal[j] = lr_adj[i];
      a.block_start[j] = blocks;
      const int64_t nb = (numel[i] + kMTChunk - 1) / kMTChunk;
      if (blocks + nb > (1ll << 30)) return fail(GNS_ERR_UNSUPPORTED, "tensor list too large");
      blocks += static_cast<int>(nb);
    }
    a.block_start[a.count] = blocks;
    if (blocks == 0) continue;
    launch_muon_apply(blocks, st, a, p_dtype, o_dtype, decay, apply_decay ? 1 : 0);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "muon apply kernel");
  return GNS_OK;
}

size_t gns_dion3_select_workspace_size(int64_t batch, int64_t rows) {
  return static_cast<size_t>(batch * rows) * sizeof(float) + 256;
}

}  // extern "C"

namespace gns {
namespace {

MatPtrs contiguous_table(const void* base) {
  MatPtrs t{};
  t.base[0] = const_cast<void*>(base);
  t.count = 0;
  return t;
}

MatPtrs list_table(const void* const* ptrs, int64_t off, int64_t n) {
  MatPtrs t{};
  for (int64_t j = 0; j < n; ++j) t.base[j] = const_cast<void*>(ptrs[off + j]);
  t.count = static_cast<int>(n);
  return t;
}

// Row selection over `count` matrices addressed by the tables (momentum, gradient,
// parameter): row norms into `norms`, top-k (or every row), gather + decay.
void launch_select(int dtype, int64_t count, int64_t rows, int64_t cols, const MatPtrs& mt, const MatPtrs& gt,
                   const MatPtrs& pt, int64_t selected, float decay, float parameter_decay, int vec,
                   __nv_bfloat16* sel, int64_t* indices_out, float* norms, cudaStream_t st) {
  const int64_t nrows = count * rows;
  dion3_momentum_rownorm_kernel<<<blocks_for(nrows, kRowThreads / 32), kRowThreads, 0, st>>>(
      mt, gt, pt, dtype, rows, nrows, cols, parameter_decay, vec, norms);
  if (selected == rows) {
    iota_kernel<<<std::min<int64_t>(blocks_for(nrows, 256), 4096), 256, 0, st>>>(indices_out, count, rows);
  } else {
    dion3_topk_kernel<<<static_cast<unsigned>(count), kSelThreads, 0, st>>>(norms, rows, selected, indices_out);
  }
  const int64_t nsel = count * selected;
  if (cols > 0)
    dion3_gather_decay_kernel<<<blocks_for(nsel, kRowThreads / 32), kRowThreads, 0, st>>>(
        mt, dtype, rows, cols, selected, nsel, indices_out, decay, vec, sel);
}

int check_select_args(int dtype, int64_t batch, int64_t rows, int64_t cols, int64_t selected, bool have_m,
                      bool have_g, bool have_p, float parameter_decay, const void* sel, const int64_t* idx,
                      void* workspace, size_t workspace_bytes) {
  if (dtype < 0 || dtype > 2) return fail(GNS_ERR_ARGUMENT, "bad dtype");
  if (batch < 0 || rows < 0 || cols < 0) return fail(GNS_ERR_ARGUMENT, "negative dimension");
  if (batch == 0 || rows == 0) return GNS_OK;
  if (selected < 1 || selected > rows) return fail(GNS_ERR_ARGUMENT, "selected must be in [1, rows]");
  if (!have_m || !have_g || idx == nullptr || sel == nullptr) return fail(GNS_ERR_ARGUMENT, "null tensor");
  if (parameter_decay != 1.0f && !have_p) return fail(GNS_ERR_ARGUMENT, "decay needs a parameter");
  if (batch > 65535) return fail(GNS_ERR_UNSUPPORTED, "batch above 65535");
  const size_t need = static_cast<size_t>(batch * rows) * sizeof(float);
  if (workspace == nullptr || workspace_bytes < need) return fail(GNS_ERR_WORKSPACE, "select workspace too small");
  return check_device();
}

// NorMuon statistics, per-matrix totals and the rescaled row update over `count`
// matrices (parameters and variances addressed by the tables).
void launch_normalize_apply(int p_dtype, int u_dtype, int64_t count, int64_t rows, int64_t cols, int64_t selected,
                            const MatPtrs& pt, const void* update, int64_t u_bstride, int64_t u_rstride,
                            const MatPtrs& vt, const int64_t* indices, float beta2, float eps, float pdecay,
                            float lr_adj, int uvec, int pvec, float* stats, float* totals, cudaStream_t st) {
  if (pdecay != 1.0f) {
    const int64_t per = rows * cols;
    const int64_t bx = std::max<int64_t>(1, std::min<int64_t>(blocks_for(per, 256),
                                                              (8 * device_sm_count() + count - 1) / count));
    decay_kernel<<<dim3(static_cast<unsigned>(bx), static_cast<unsigned>(count)), 256, 0, st>>>(pt, p_dtype, per,
                                                                                                   pdecay);
  }
  if (selected == 0 || cols == 0) return;
  const int64_t nsel = count * selected;
  dion3_rowstats_kernel<<<blocks_for(nsel, kRowThreads / 32), kRowThreads, 0, st>>>(
      update, u_dtype, u_bstride, u_rstride, rows, cols, selected, nsel, indices, vt, beta2, eps, uvec, stats);
  dion3_totals_kernel<<<static_cast<unsigned>(count), 256, 0, st>>>(stats, selected, eps, totals);
  dion3_apply_kernel<<<blocks_for(nsel, kRowThreads / 32), kRowThreads, 0, st>>>(
      pt, p_dtype, update, u_dtype, u_bstride, u_rstride, rows, cols, selected, nsel, indices, stats, totals, lr_adj,
      pvec);
}

int check_normalize_args(int p_dtype, int u_dtype, int64_t batch, int64_t rows, int64_t cols, int64_t selected,
                         bool have_p, bool have_v, const void* update, const int64_t* indices, size_t workspace_bytes,
                         const void* workspace) {
  if (p_dtype < 0 || p_dtype > 2 || u_dtype < 0 || u_dtype > 2) return fail(GNS_ERR_ARGUMENT, "bad dtype");
  if (batch < 0 || rows < 0 || cols < 0 || selected < 0) return fail(GNS_ERR_ARGUMENT, "negative dimension");
  if (selected > rows) return fail(GNS_ERR_ARGUMENT, "selected > rows");
  if (batch == 0 || rows == 0) return GNS_OK;
  if (!have_p || !have_v || (selected > 0 && (update == nullptr || indices == nullptr)))
    return fail(GNS_ERR_ARGUMENT, "null tensor");
  if (batch > 65535) return fail(GNS_ERR_UNSUPPORTED, "batch above 65535");
  const size_t need = static_cast<size_t>(batch * selected * 3 + batch * 2) * sizeof(float) + 256;
  if (workspace == nullptr || workspace_bytes < need) return fail(GNS_ERR_WORKSPACE, "normalize workspace too small");
  return check_device();
}

float* totals_after(float* stats, int64_t batch, int64_t selected) {
  return reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(stats + batch * selected * 3) + 255) & ~uintptr_t(255));
}

}  // namespace
}  // namespace gns

extern "C" {

int gns_dion3_select_rows(int dtype, int64_t batch, int64_t rows, int64_t cols, void* momentum, const void* gradient,
                          void* parameter, int64_t selected, float decay, float parameter_decay,
                          void* selected_out_bf16, int64_t* indices_out, void* workspace, size_t workspace_bytes,
                          gns_stream_t stream) {
  clear_error();
  int rc = check_select_args(dtype, batch, rows, cols, selected, momentum != nullptr, gradient != nullptr,
                             parameter != nullptr, parameter_decay, selected_out_bf16, indices_out, workspace,
                             workspace_bytes);
  if (rc != GNS_OK || batch == 0 || rows == 0) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t es = dtype_size(dtype);
  const int vec = (cols % 8 == 0) && ((cols * es) % 16 == 0) && al16(momentum) && al16(gradient) &&
                  (parameter == nullptr || al16(parameter)) && al16(selected_out_bf16);
  launch_select(dtype, batch, rows, cols, contiguous_table(momentum), contiguous_table(gradient),
                contiguous_table(parameter), selected, decay, parameter_decay, vec,
                static_cast<__nv_bfloat16*>(selected_out_bf16), indices_out, static_cast<float*>(workspace), st);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "dion3 select kernels");
  return GNS_OK;
}

int gns_dion3_select_rows_multi(int dtype, int count, int64_t rows, int64_t cols, void* const* momenta,
                                const void* const* gradients, void* const* parameters, int64_t selected, float decay,
                                float parameter_decay, void* selected_out_bf16, int64_t* indices_out, void* workspace,
                                size_t workspace_bytes, gns_stream_t stream) {
  clear_error();
  if (count < 0) return fail(GNS_ERR_ARGUMENT, "negative count");
  bool have_m = momenta != nullptr, have_g = gradients != nullptr, have_p = parameters != nullptr;
  for (int i = 0; i < count; ++i) {
    have_m = have_m && momenta[i] != nullptr;
    have_g = have_g && gradients[i] != nullptr;
    have_p = have_p && parameters[i] != nullptr;
  }
  int rc = check_select_args(dtype, count, rows, cols, selected, have_m, have_g, have_p, parameter_decay,
                             selected_out_bf16, indices_out, workspace, workspace_bytes);
  if (rc != GNS_OK || count == 0 || rows == 0) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t es = dtype_size(dtype);
  int vec = (cols % 8 == 0) && ((cols * es) % 16 == 0) && al16(selected_out_bf16);
  for (int i = 0; i < count && vec; ++i)
    vec = al16(momenta[i]) && al16(gradients[i]) && (!have_p || al16(parameters[i]));
  float* norms = static_cast<float*>(workspace);
  auto* sel = static_cast<__nv_bfloat16*>(selected_out_bf16);
  for (int64_t off = 0; off < count; off += kD3) {
    const int64_t n = std::min<int64_t>(kD3, count - off);
    const MatPtrs pt = have_p ? list_table(parameters, off, n) : contiguous_table(nullptr);
    launch_select(dtype, n, rows, cols, list_table(momenta, off, n), list_table(gradients, off, n), pt, selected,
                  decay, parameter_decay, vec, sel + off * selected * cols, indices_out + off * selected,
                  norms + off * rows, st);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "dion3 select kernels");
  return GNS_OK;
}

size_t gns_dion3_normalize_workspace_size(int64_t batch, int64_t selected) {
  return static_cast<size_t>(batch * selected * 3 + batch * 2) * sizeof(float) + 512;
}

int gns_dion3_normalize_apply(int p_dtype, int u_dtype, int64_t batch, int64_t rows, int64_t cols, int64_t selected,
                              void* parameter, const void* update, int64_t u_bstride, int64_t u_rstride,
                              float* variance, const int64_t* indices, float beta2, float eps, float lr, float wd,
                              float lr_adj, void* workspace, size_t workspace_bytes, gns_stream_t stream) {
  clear_error();
  int rc = check_normalize_args(p_dtype, u_dtype, batch, rows, cols, selected, parameter != nullptr,
                                variance != nullptr, update, indices, workspace_bytes, workspace);
  if (rc != GNS_OK || batch == 0 || rows == 0) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t pes = dtype_size(p_dtype), ues = dtype_size(u_dtype);
  const int uvec = (cols % 8 == 0) && al16(update) && ((u_rstride * ues) % 16 == 0) &&
                   (batch == 1 || (u_bstride * ues) % 16 == 0);
  const int pvec = uvec && al16(parameter) && ((cols * pes) % 16 == 0);
  float* stats = static_cast<float*>(workspace);
  launch_normalize_apply(p_dtype, u_dtype, batch, rows, cols, selected, contiguous_table(parameter), update,
                         u_bstride, u_rstride, contiguous_table(variance), indices, beta2, eps, 1.0f - lr * wd,
                         lr_adj, uvec, pvec, stats, totals_after(stats, batch, selected), st);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "dion3 normalize kernels");
  return GNS_OK;
}

int gns_dion3_normalize_apply_multi(int p_dtype, int u_dtype, int count, int64_t rows, int64_t cols,
                                    int64_t selected, void* const* parameters, const void* update, int64_t u_bstride,
                                    int64_t u_rstride, float* const* variances, const int64_t* indices, float beta2,
                                    float eps, float lr, float wd, float lr_adj, void* workspace,
                                    size_t workspace_bytes, gns_stream_t stream) {
  clear_error();
  if (count < 0) return fail(GNS_ERR_ARGUMENT, "negative count");
  bool have_p = parameters != nullptr, have_v = variances != nullptr;
  for (int i = 0; i < count; ++i) {
    have_p = have_p && parameters[i] != nullptr;
    have_v = have_v && variances[i] != nullptr;
  }
  int rc = check_normalize_args(p_dtype, u_dtype, count, rows, cols, selected, have_p, have_v, update, indices,
                                workspace_bytes, workspace);
  if (rc != GNS_OK || count == 0 || rows == 0) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t pes = dtype_size(p_dtype), ues = dtype_size(u_dtype);
  const int uvec = (cols % 8 == 0) && al16(update) && ((u_rstride * ues) % 16 == 0) &&
                   (count == 1 || (u_bstride * ues) % 16 == 0);
  int pvec = uvec && ((cols * pes) % 16 == 0);
  for (int i = 0; i < count && pvec; ++i) pvec = al16(parameters[i]);
  float* stats = static_cast<float*>(workspace);
  float* totals = totals_after(stats, count, selected);
  const auto* u = static_cast<const char*>(update);
  for (int64_t off = 0; off < count; off += kD3) {
    const int64_t n = std::min<int64_t>(kD3, count - off);
    const void* const* vptrs = reinterpret_cast<const void* const*>(variances);
    launch_normalize_apply(p_dtype, u_dtype, n, rows, cols, selected, list_table(parameters, off, n),
                           u + off * u_bstride * ues, u_bstride, u_rstride, list_table(vptrs, off, n),
                           indices + off * selected, beta2, eps, 1.0f - lr * wd, lr_adj, uvec, pvec,
                           stats + off * selected * 3, totals + off * 2, st);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "dion3 normalize kernels");
  return GNS_OK;
}

int gns_dion3_normalize_rows(int u_dtype, int64_t batch, int64_t rows, int64_t cols, int64_t selected,
                             const void* update, int64_t u_bstride, int64_t u_rstride, float* variance,
                             const int64_t* indices, float beta2, float eps, float* normalized, float* squared_norms,
                             void* workspace, size_t workspace_bytes, gns_stream_t stream) {
  clear_error();
  if (u_dtype < 0 || u_dtype > 2) return fail(GNS_ERR_ARGUMENT, "bad dtype");
  if (batch < 0 || rows < 0 || cols < 0 || selected < 0) return fail(GNS_ERR_ARGUMENT, "negative dimension");
  if (selected > rows) return fail(GNS_ERR_ARGUMENT, "selected > rows");
  if (batch == 0) return GNS_OK;
  if (squared_norms == nullptr || variance == nullptr) return fail(GNS_ERR_ARGUMENT, "null tensor");
  if (batch > 65535) return fail(GNS_ERR_UNSUPPORTED, "batch above 65535");
  int rc = check_device();
  if (rc != GNS_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (selected == 0 || cols == 0) {
    cudaError_t e = cudaMemsetAsync(squared_norms, 0, static_cast<size_t>(batch) * 2 * sizeof(float), st);
    return e == cudaSuccess ? GNS_OK : cuda_fail(e, "zero squared norms");
  }
  if (update == nullptr || indices == nullptr || normalized == nullptr) return fail(GNS_ERR_ARGUMENT, "null tensor");
  const size_t need = static_cast<size_t>(batch * selected * 3) * sizeof(float);
  if (workspace == nullptr || workspace_bytes < need) return fail(GNS_ERR_WORKSPACE, "normalize workspace too small");
  float* stats = static_cast<float*>(workspace);
  const int64_t nsel = batch * selected;
  const int64_t ues = dtype_size(u_dtype);
  const int uvec = (cols % 8 == 0) && al16(update) && ((u_rstride * ues) % 16 == 0) &&
                   (batch == 1 || (u_bstride * ues) % 16 == 0);
  dion3_rowstats_kernel<<<blocks_for(nsel, kRowThreads / 32), kRowThreads, 0, st>>>(
      update, u_dtype, u_bstride, u_rstride, rows, cols, selected, nsel, indices, contiguous_table(variance), beta2,
      eps, uvec, stats);
  dion3_write_normalized_kernel<<<blocks_for(nsel, kRowThreads / 32), kRowThreads, 0, st>>>(
      update, u_dtype, u_bstride, u_rstride, rows, cols, selected, nsel, indices, stats, normalized);
  dion3_sums_kernel<<<static_cast<unsigned>(batch), 256, 0, st>>>(stats, selected, squared_norms);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GNS_OK : cuda_fail(e, "dion3 normalize-rows kernels");
}

int gns_dion3_apply_rows(int p_dtype, int64_t batch, int64_t rows, int64_t cols, int64_t selected, void* parameter,
                         const float* normalized, const int64_t* indices, const float* squared_norms, float lr,
                         float wd, float lr_adj, float eps, gns_stream_t stream) {
  clear_error();
  if (p_dtype < 0 || p_dtype > 2) return fail(GNS_ERR_ARGUMENT, "bad dtype");
  if (batch < 0 || rows < 0 || cols < 0 || selected < 0) return fail(GNS_ERR_ARGUMENT, "negative dimension");
  if (selected > rows) return fail(GNS_ERR_ARGUMENT, "selected > rows");
  if (batch == 0 || rows == 0) return GNS_OK;
  if (parameter == nullptr) return fail(GNS_ERR_ARGUMENT, "null parameter");
  if (selected > 0 && (normalized == nullptr || indices == nullptr || squared_norms == nullptr))
    return fail(GNS_ERR_ARGUMENT, "null tensor");
  int rc = check_device();
  if (rc != GNS_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float pdecay = 1.0f - lr * wd;
  const MatPtrs pt = contiguous_table(parameter);
  if (pdecay != 1.0f) {
    const int64_t per = rows * cols;
    const int64_t bx = std::max<int64_t>(1, std::min<int64_t>(blocks_for(per, 256),
                                                              (8 * device_sm_count() + batch - 1) / batch));
    decay_kernel<<<dim3(static_cast<unsigned>(bx), static_cast<unsigned>(batch)), 256, 0, st>>>(pt, p_dtype, per,
                                                                                                   pdecay);
  }
  if (selected > 0 && cols > 0) {
    const int64_t nsel = batch * selected;
    dion3_apply_normalized_kernel<<<blocks_for(nsel, kRowThreads / 32), kRowThreads, 0, st>>>(
        pt, p_dtype, normalized, rows, cols, selected, nsel, indices, squared_norms, lr_adj, eps);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GNS_OK : cuda_fail(e, "dion3 apply-rows kernels");
}

int gns_adamw_step(int count, void* const* params, const void* const* grads, void* const* exp_avgs,
                   void* const* exp_avg_sqs, const int64_t* numel, int p_dtype, int g_dtype, int s_dtype,
                   const float* lr_bc1, const float* inv_bc2, float beta1, float beta2, float one_minus_beta1,
                   float one_minus_beta2, float epsilon, float decay, int apply_decay, gns_stream_t stream) {
  clear_error();
  if (count < 0 || (count > 0 && (params == nullptr || grads == nullptr || exp_avgs == nullptr ||
                                  exp_avg_sqs == nullptr || numel == nullptr || lr_bc1 == nullptr ||
                                  inv_bc2 == nullptr)))
    return fail(GNS_ERR_ARGUMENT, "bad tensor list");
  for (int dt : {p_dtype, g_dtype, s_dtype})
    if (dt < 0 || dt > 2) return fail(GNS_ERR_ARGUMENT, "bad dtype");
  if (count == 0) return GNS_OK;
  int rc = check_device();
  if (rc != GNS_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const AdamWScalars k{beta1, one_minus_beta1, beta2, one_minus_beta2, epsilon, decay, apply_decay ? 1 : 0};
  for (int off = 0; off < count; off += kMT4) {
    MT4Args a{};
    const int blocks = fill_mt4(a, off, count, grads, params, exp_avgs, exp_avg_sqs, numel, lr_bc1, inv_bc2, &rc);
    if (rc != GNS_OK) return rc;
    if (blocks == 0) continue;
    adamw_kernel<<<blocks, kMTThreads, 0, st>>>(a, g_dtype, p_dtype, s_dtype, k);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GNS_OK : cuda_fail(e, "adamw kernel");
}

int gns_lion_step(int count, void* const* params, const void* const* grads, void* const* buffers, const int64_t* numel,
                  int p_dtype, int g_dtype, int s_dtype, float lr, float beta1, float beta2, float one_minus_beta1,
                  float one_minus_beta2, float decay, int apply_decay, gns_stream_t stream) {
  clear_error();
  if (count < 0 || (count > 0 && (params == nullptr || grads == nullptr || buffers == nullptr || numel == nullptr)))
    return fail(GNS_ERR_ARGUMENT, "bad tensor list");
  for (int dt : {p_dtype, g_dtype, s_dtype})
    if (dt < 0 || dt > 2) return fail(GNS_ERR_ARGUMENT, "bad dtype");
  if (count == 0) return GNS_OK;
  int rc = check_device();
  if (rc != GNS_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const LionScalars k{beta1, one_minus_beta1, beta2, one_minus_beta2, lr, decay, apply_decay ? 1 : 0};
  for (int off = 0; off < count; off += kMT4) {
    MT4Args a{};
    const int blocks = fill_mt4(a, off, count, grads, params, buffers, nullptr, numel, nullptr, nullptr, &rc);
    if (rc != GNS_OK) return rc;
    if (blocks == 0) continue;
    lion_kernel<<<blocks, kMTThreads, 0, st>>>(a, g_dtype, p_dtype, s_dtype, k);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GNS_OK : cuda_fail(e, "lion kernel");
}

}  // extern "C"
