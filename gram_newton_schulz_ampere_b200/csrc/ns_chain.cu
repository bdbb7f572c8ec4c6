// Frobenius normalisation kernels and the Gram / standard Newton-Schulz chains.
//
// The chains keep every intermediate in a caller-provided workspace, in fp16
// with 16-byte aligned row pitch, so each product is a TMA-fed tcgen05 GEMM:
//   Gram:      G = X X^T (wide) or X^T X (tall), symmetric, upper tiles only
// Every symmetric m x m intermediate (G, P, GP, Q) is stored as its upper block
// triangle (256 x 256 blocks); products read the missing tiles transposed.
//   iteration: P = c G G + b G;  Q = P + a I (fused second output) or Q = Q P + a Q;
//              GP = G P + a G;   G = P GP + a GP
//   reset:     X = Q X (wide) or X Q (tall), then a fresh Gram
//   output:    Q X (wide) or X Q (tall), rounded through fp16 then to the caller's dtype
// Wide/tall orientation is expressed purely through operand strides; the GEMM
// reads transposed views with MN-major shared-memory descriptors.
#include <atomic>
#include <mutex>
#include <string>
#include <type_traits>

#include "../../include/gns_b200.h"
#include "gns_common.cuh"
#include "gns_host.h"

namespace gns {

// Set by the normalisation kernel when its bounded wait gives up.
__device__ int g_norm_status = 0;
constexpr int kNormTimeout = 4;

namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ float block_sum_deterministic(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  if (threadIdx.x < 32) {
    t = (lane < static_cast<int>(blockDim.x >> 5)) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  __syncthreads();
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

// 8 consecutive elements as fp32, from a 16-byte (16-bit types) or 2x16-byte (fp32) load.
__device__ __forceinline__ void load8(const void* base, int64_t idx, int dtype, float (&f)[8]) {
  if (dtype == kF32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
    float4 a = p[0], b = p[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + idx);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 t;
      if (dtype == kBF16)
        t = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[e]));
      else
        t = __half22float2(*reinterpret_cast<__half2*>(&w[e]));
      f[2 * e] = t.x;
      f[2 * e + 1] = t.y;
    }
  }
}

// Element offset of 8-element vector `tu` of a row slice starting at `first`
// (the slice's first element): rows of `cv` vectors, `rstride` apart. A slice
// whose rows are adjacent (rstride == 8 cv) is one run and needs no division.
struct SliceIndex {
  int64_t first, rstride;
  uint32_t cv;
  bool flat;
  __device__ __forceinline__ int64_t operator()(uint32_t tu) const {
    return flat ? first + static_cast<int64_t>(tu) * 8
                : first + static_cast<int64_t>(tu / cv) * rstride + static_cast<int64_t>(tu % cv) * 8;
  }
};

// Sum of squares of this CTA's row slice [r0, r1) of matrix `b`.
__device__ __forceinline__ float slice_sumsq(const void* __restrict__ x, int dtype, int64_t cols, int64_t base,
                                             int64_t rstride, int64_t r0, int64_t r1, int vec) {
  float acc = 0.0f;
  if (vec) {
    // Four independent 16-byte loads per thread in flight (memory-level parallelism).
    // 32-bit slice indexing: a slice holds fewer than 2^31 vectors (checked on the host).
    const uint32_t cv = static_cast<uint32_t>(cols / 8);
    const uint32_t n = static_cast<uint32_t>((r1 - r0) * cv);
    const uint32_t step = blockDim.x;
    const SliceIndex at{base + r0 * rstride, rstride, cv, rstride == cols};
    uint32_t t = threadIdx.x;
    for (; t + 3 * step < n; t += 4 * step) {
      float f[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) load8(x, at(t + u * step), dtype, f[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc = fmaf(f[u][e], f[u][e], acc);
    }
    for (; t < n; t += step) {
      float f[8];
      load8(x, at(t), dtype, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaf(f[e], f[e], acc);
    }
  } else {
    const int64_t n = (r1 - r0) * cols;
    for (int64_t t = threadIdx.x; t < n; t += blockDim.x) {
      const int64_t r = r0 + t / cols, c = t % cols;
      const float f = load_as_float(x, base + r * rstride + c, dtype);
      acc = fmaf(f, f, acc);
    }
  }
  return acc;
}

__device__ __forceinline__ void scale_slice_to_half(const void* __restrict__ x, int dtype, int64_t cols, int64_t base,
                                                    int64_t rstride, int64_t r0, int64_t r1, int vec, float denom,
                                                    __half* __restrict__ out, int64_t obase, int64_t out_ld);

// One pass over HBM: CTA (p, b) sums the squares of its row slice, publishes the
// partial, waits (bounded) until `arrive_target` slices of matrix b have arrived
// (every slice: gridDim.x), then rescales its own slice (now L2-resident) to fp16:
//   out = fp16(x / (sqrt(sum of partials) + eps)), partials summed in a fixed order.
// CTAs of one matrix are consecutive in launch order and few enough to be
// co-resident; a wait that exceeds `wait_limit_ns` records kNormTimeout and
// fills the CTA's slice of the output with NaN, so that a result computed from
// it downstream is visibly invalid rather than plausibly wrong.
__global__ void __launch_bounds__(kNormThreads) normalize_fused_kernel(
    const void* __restrict__ x, int dtype, int64_t rows, int64_t cols, int64_t bstride, int64_t rstride,
    int64_t rows_per_part, int vec, float* __restrict__ partial, unsigned int* __restrict__ arrived, float eps,
    __half* __restrict__ out, int64_t out_ld, unsigned int arrive_target, unsigned long long wait_limit_ns) {
  __shared__ float red[32];
  __shared__ int s_abort;
  const int b = blockIdx.y, p = blockIdx.x;
  const int parts = gridDim.x;
  pdl_launch_dependents();
  pdl_wait_predecessor();
  // Clamped so that a slice past the last row is empty (r1 - r0 == 0), never negative.
  const int64_t r0 = min(rows, p * rows_per_part);
  const int64_t r1 = min(rows, r0 + rows_per_part);
  const int64_t base = static_cast<int64_t>(b) * bstride;
  const float mine = block_sum_deterministic(slice_sumsq(x, dtype, cols, base, rstride, r0, r1, vec), red);
  if (threadIdx.x == 0) {
    partial[static_cast<int64_t>(b) * parts + p] = mine;
    __threadfence();
    atomicAdd(&arrived[b], 1u);
    int abort = 0;
    volatile unsigned int* flag = &arrived[b];
    if (*flag < arrive_target) {
      const unsigned long long start = global_timer_ns();
      while (*flag < arrive_target) {
        if (global_timer_ns() - start > wait_limit_ns) {
          abort = 1;
          atomicCAS(&g_norm_status, 0, kNormTimeout);
          break;
        }
        __nanosleep(200);
      }
    }
    __threadfence();
    s_abort = abort;
  }
  __syncthreads();
  if (s_abort) {
    const __half nan = __ushort_as_half(static_cast<unsigned short>(0x7E00));
    const int64_t n = (r1 - r0) * cols;
    __half* o = out + static_cast<int64_t>(b) * rows * out_ld;
    for (int64_t t = threadIdx.x; t < n; t += blockDim.x) o[(r0 + t / cols) * out_ld + t % cols] = nan;
    return;
  }
  float t0 = 0.0f;
  for (int q = threadIdx.x; q < parts; q += blockDim.x) t0 += *reinterpret_cast<volatile float*>(&partial[static_cast<int64_t>(b) * parts + q]);
  const float total = block_sum_deterministic(t0, red);
  const float denom = sqrtf(total) + eps;
  scale_slice_to_half(x, dtype, cols, base, rstride, r0, r1, vec, denom, out, static_cast<int64_t>(b) * rows * out_ld,
                      out_ld);
}

// out[b] = fp16(x[b] / (sqrt(sumsq[b]) + eps)) for a norm computed elsewhere
// (gns_frobenius_scale: the column-sharded path sums the squares over ranks first).
__global__ void __launch_bounds__(kNormThreads) scale_with_sumsq_kernel(
    const void* __restrict__ x, int dtype, int64_t rows, int64_t cols, int64_t bstride, int64_t rstride,
    int64_t rows_per_part, int vec, const float* __restrict__ sumsq, float eps, __half* __restrict__ out,
    int64_t out_ld) {
  const int b = blockIdx.y, p = blockIdx.x;
  const int64_t r0 = min(rows, p * rows_per_part);
  const int64_t r1 = min(rows, r0 + rows_per_part);
  const float denom = sqrtf(sumsq[b]) + eps;
  scale_slice_to_half(x, dtype, cols, static_cast<int64_t>(b) * bstride, rstride, r0, r1, vec, denom, out,
                      static_cast<int64_t>(b) * rows * out_ld, out_ld);
}

// partial[b * gridDim.x + p] = sum of squares of row slice p of matrix b.
__global__ void __launch_bounds__(kNormThreads) sumsq_slices_kernel(const void* __restrict__ x, int dtype,
                                                                    int64_t rows, int64_t cols, int64_t bstride,
                                                                    int64_t rstride, int64_t rows_per_part, int vec,
                                                                    float* __restrict__ partial) {
  __shared__ float red[32];
  const int b = blockIdx.y, p = blockIdx.x;
  const int64_t r0 = min(rows, p * rows_per_part);
  const int64_t r1 = min(rows, r0 + rows_per_part);
  const float s = block_sum_deterministic(
      slice_sumsq(x, dtype, cols, static_cast<int64_t>(b) * bstride, rstride, r0, r1, vec), red);
  if (threadIdx.x == 0) partial[static_cast<int64_t>(b) * gridDim.x + p] = s;
}

// out[b] = sum of the `parts` partials of matrix b, in a fixed order.
__global__ void __launch_bounds__(kNormThreads) sumsq_reduce_kernel(const float* __restrict__ partial, int parts,
                                                                    float* __restrict__ out) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  float t = 0.0f;
  for (int q = threadIdx.x; q < parts; q += blockDim.x) t += partial[static_cast<int64_t>(b) * parts + q];
  const float s = block_sum_deterministic(t, red);
  if (threadIdx.x == 0) out[b] = s;
}

// dst[b] (fp16, ld_dst) = src[b] (fp32 or fp16 per src_f32, strides in elements), m x m.
// With src_upper the source is a symmetric matrix stored as its upper block
// triangle (kUpperBlock blocks): elements below the block diagonal are read
// from their mirror positions, so dst is the full matrix.
__global__ void cast_square_to_half_kernel(const void* __restrict__ src, int src_f32, int src_upper,
                                           int64_t s_bstride, int64_t s_ld, __half* __restrict__ dst,
                                           int64_t d_bstride, int64_t d_ld, int64_t batch, int64_t m) {
  const int64_t n = batch * m * m;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = t / (m * m), rc = t % (m * m), r = rc / m, c = rc % m;
    const bool mirrored = src_upper && (c / kUpperBlock < r / kUpperBlock);
    const int64_t si = b * s_bstride + (mirrored ? c * s_ld + r : r * s_ld + c);
    const float v = src_f32 ? static_cast<const float*>(src)[si] : __half2float(static_cast<const __half*>(src)[si]);
    dst[b * d_bstride + r * d_ld + c] = __float2half_rn(v);
  }
}

// Writes fp16(x / denom) for rows [r0, r1) of one matrix (shared by both scale kernels).
// x / d rounded to nearest-even in fp32, given rcp = 1/d rounded to nearest:
// q0 = x rcp is within one ulp of x / d, the remainder x - q0 d is exact in
// one fma, and q0 + rem rcp rounds to the correctly rounded quotient
// (Markstein's theorem for division by a correctly rounded reciprocal). Valid
// for normal quotients; a quotient in fp32's subnormal range rounds to zero in
// fp16 either way. Three instructions per element instead of a full division.
__device__ __forceinline__ float div_by(float x, float d, float rcp) {
  const float q0 = x * rcp;
  const float rem = fmaf(-q0, d, x);
  return fmaf(rem, rcp, q0);
}

__device__ __forceinline__ void scale_slice_to_half(const void* __restrict__ x, int dtype, int64_t cols, int64_t base,
                                                    int64_t rstride, int64_t r0, int64_t r1, int vec, float denom,
                                                    __half* __restrict__ out, int64_t obase, int64_t out_ld) {
  const float rcp = __frcp_rn(denom);
  if (vec) {
    // 32-bit slice indexing: a slice holds fewer than 2^31 vectors (checked on the host).
    const uint32_t cv = static_cast<uint32_t>(cols / 8);
    const uint32_t n = static_cast<uint32_t>((r1 - r0) * cv);
    const uint32_t step = blockDim.x;
    const SliceIndex src{base + r0 * rstride, rstride, cv, rstride == cols};
    const SliceIndex dst{obase + r0 * out_ld, out_ld, cv, out_ld == cols};
    auto emit = [&](uint32_t tu, const float (&f)[8]) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __half2 h = __floats2half2_rn(div_by(f[2 * e], denom, rcp), div_by(f[2 * e + 1], denom, rcp));
        w[e] = *reinterpret_cast<const uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(out + dst(tu)) = make_uint4(w[0], w[1], w[2], w[3]);
    };
    uint32_t t = threadIdx.x;
    for (; t + 3 * step < n; t += 4 * step) {
      float f[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) load8(x, src(t + u * step), dtype, f[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u) emit(t + u * step, f[u]);
    }
    for (; t < n; t += step) {
      float f[8];
      load8(x, src(t), dtype, f);
      emit(t, f);
    }
  } else {
    const int64_t n = (r1 - r0) * cols;
    for (int64_t t = threadIdx.x; t < n; t += blockDim.x) {
      const int64_t r = r0 + t / cols, c = t % cols;
      out[obase + r * out_ld + c] = __float2half_rn(div_by(load_as_float(x, base + r * rstride + c, dtype), denom, rcp));
    }
  }
}

// out[b][r][c] = cast(x[b][r][c]) for fp16 x; used when a chain has no products.
// out[b][r][c] = x[b][r][c] (fp16 workspace, row pitch ldx, a multiple of 8) in
// out_dtype: a CTA per row, eight columns per thread with 16-byte loads (and
// 16-byte stores when out_vec: output base and strides 16-byte aligned).
__global__ void cast_from_half_kernel(const __half* __restrict__ x, int64_t ldx, int64_t batch, int64_t rows,
                                      int64_t cols, void* out, int out_dtype, int64_t obstride, int64_t orstride,
                                      int out_vec) {
  const int64_t nrows = batch * rows;
  const int64_t groups = (cols + 7) / 8;
  for (int64_t row = blockIdx.x; row < nrows; row += gridDim.x) {
    const int64_t b = row / rows, r = row - b * rows;
    const __half* src = x + row * ldx;
    const int64_t obase = b * obstride + r * orstride;
    for (int64_t g = threadIdx.x; g < groups; g += blockDim.x) {
      const int64_t c = g * 8;
      if (c + 8 <= cols) {
        const uint4 u = *reinterpret_cast<const uint4*>(src + c);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
        float f[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
          f[2 * k] = p.x;
          f[2 * k + 1] = p.y;
        }
        if (out_vec && out_dtype == kF32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + obase + c);
          dst[0] = make_float4(f[0], f[1], f[2], f[3]);
          dst[1] = make_float4(f[4], f[5], f[6], f[7]);
        } else if (out_vec && out_dtype == kBF16) {
          uint32_t o[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
            o[k] = *reinterpret_cast<const uint32_t*>(&h);
          }
          *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + obase + c) = make_uint4(o[0], o[1], o[2], o[3]);
        } else if (out_vec) {
          *reinterpret_cast<uint4*>(static_cast<__half*>(out) + obase + c) = u;
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) store_from_float(out, obase + c + k, out_dtype, f[k]);
        }
      } else {
        for (int64_t k = c; k < cols; ++k) store_from_float(out, obase + k, out_dtype, __half2float(src[k]));
      }
    }
  }
}

int norm_parts(int64_t batch, int64_t rows) {
  const int64_t sms = static_cast<int64_t>(device_sm_count());
  int64_t parts = (4 * sms + batch - 1) / batch;
  if (parts > 2 * sms) parts = 2 * sms;  // every slice of a matrix must be co-resident
  if (parts > rows) parts = rows;
  if (parts < 1) parts = 1;
  if (parts > 4096) parts = 4096;
  return static_cast<int>(parts);
}

}  // namespace

int normalize_status(int* status, int clear) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_norm_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "read normalize status");
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_norm_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "clear normalize status");
  }
  return GNS_OK;
}

size_t normalize_workspace_bytes(int64_t batch, int64_t rows, int64_t /*cols*/) {
  // Partial sums (at most 4096 per matrix) + one arrival counter per matrix.
  const int64_t parts = rows < 4096 ? (rows < 1 ? 1 : rows) : 4096;
  return static_cast<size_t>(batch * parts) * sizeof(float) + static_cast<size_t>(batch) * sizeof(unsigned int) + 512;
}

// Wall-clock limit of the normalisation's arrival wait (gns_set_wait_limit_ns).
std::atomic<unsigned long long> g_norm_wait_limit_ns{kWaitLimitNs};

int launch_normalize(int x_dtype, int64_t batch, int64_t rows, int64_t cols, const void* x, int64_t x_bstride,
                     int64_t x_rstride, void* out, int64_t out_ld, float eps, void* workspace, size_t workspace_bytes,
                     cudaStream_t stream, unsigned int extra_arrivals) {
  if (x_dtype < 0 || x_dtype > 2) return fail(GNS_ERR_ARGUMENT, "bad input dtype");
  if (batch < 0 || rows < 0 || cols < 0) return fail(GNS_ERR_ARGUMENT, "negative dimension");
  if (out_ld < cols) return fail(GNS_ERR_ARGUMENT, "out_ld < cols");
  if (batch == 0 || rows == 0 || cols == 0) return GNS_OK;
  if (batch > 65535) return fail(GNS_ERR_UNSUPPORTED, "batch above 65535");
  const int parts = norm_parts(batch, rows);
  const size_t partial_bytes = static_cast<size_t>(batch * parts) * sizeof(float);
  const size_t counter_off = (partial_bytes + 255) & ~size_t(255);
  const size_t need = counter_off + static_cast<size_t>(batch) * sizeof(unsigned int);
  if (workspace == nullptr || workspace_bytes < need) return fail(GNS_ERR_WORKSPACE, "normalize workspace too small");
  const int64_t rpp = (rows + parts - 1) / parts;
  if (rpp * ((cols + 7) / 8) >= (int64_t(1) << 31)) return fail(GNS_ERR_UNSUPPORTED, "matrix slice too large");
  const int64_t es = dtype_size(x_dtype);
  const int vec = (cols % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((x_rstride * es) % 16 == 0) &&
                  (batch == 1 || (x_bstride * es) % 16 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0) &&
                  (out_ld % 8 == 0);
  float* partial = static_cast<float*>(workspace);
  unsigned int* arrived = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(workspace) + counter_off);
  cudaError_t me = cudaMemsetAsync(arrived, 0, static_cast<size_t>(batch) * sizeof(unsigned int), stream);
  if (me != cudaSuccess) return cuda_fail(me, "normalize counter reset");
  // Launch only non-empty slices: ceil(rows / rpp) <= parts.
  const int used_parts = static_cast<int>((rows + rpp - 1) / rpp);
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(used_parts, static_cast<unsigned>(batch));
  cfg.blockDim = dim3(kNormThreads);
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, normalize_fused_kernel, x, x_dtype, rows, cols, x_bstride, x_rstride, rpp,
                                     vec, partial, arrived, eps, static_cast<__half*>(out), out_ld,
                                     static_cast<unsigned int>(used_parts) + extra_arrivals,
                                     g_norm_wait_limit_ns.load());
  if (e != cudaSuccess) return cuda_fail(e, "normalize kernel launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "normalize kernels");
  return GNS_OK;
}

namespace {

// Workspace layout of a chain; identical code sizes it (Sizer) and carves it (Carver).
struct ChainBuffers {
  void* norm_ws = nullptr;
  size_t norm_ws_bytes = 0;
  __half* x[2] = {nullptr, nullptr};
  __half* g = nullptr;
  __half* p = nullptr;
  __half* gp = nullptr;
  __half* q[2] = {nullptr, nullptr};
  int64_t ldx = 0, ldm = 0, xb = 0, mb = 0;
};

template <class Alloc>
void layout_chain(Alloc& al, ChainBuffers* cb, int64_t batch, int64_t rows, int64_t cols, bool gram) {
  const int64_t m = rows < cols ? rows : cols;
  const int64_t ldx = round_up(cols, 8), ldm = round_up(m, 8);
  const int64_t xb = rows * ldx, mb = m * ldm;
  const size_t xbytes = static_cast<size_t>(batch * xb) * 2, mbytes = static_cast<size_t>(batch * mb) * 2;
  const size_t nbytes = normalize_workspace_bytes(batch, rows, cols);
  auto take = [&](size_t bytes) -> void* {
    if constexpr (std::is_same<Alloc, Carver>::value) {
      return al.take(bytes);
    } else {
      al.take(bytes);
      return nullptr;
    }
  };
  void* nws = take(nbytes);
  void* x0 = take(xbytes);
  void* x1 = take(xbytes);
  void* g = take(mbytes);
  void* p = take(mbytes);
  void* gp = gram ? take(mbytes) : nullptr;
  void* q0 = gram ? take(mbytes) : nullptr;
  void* q1 = gram ? take(mbytes) : nullptr;
  if (cb) {
    cb->norm_ws = nws;
    cb->norm_ws_bytes = nbytes;
    cb->x[0] = static_cast<__half*>(x0);
    cb->x[1] = static_cast<__half*>(x1);
    cb->g = static_cast<__half*>(g);
    cb->p = static_cast<__half*>(p);
    cb->gp = static_cast<__half*>(gp);
    cb->q[0] = static_cast<__half*>(q0);
    cb->q[1] = static_cast<__half*>(q1);
    cb->ldx = ldx;
    cb->ldm = ldm;
    cb->xb = xb;
    cb->mb = mb;
  }
}

struct Chain {
  int64_t batch, rows, cols, m, n;
  bool tall;
  ChainBuffers buf;
  cudaStream_t stream;
  bool reverse = false;

  // Launches one product; consecutive products walk the batch in alternating
  // directions so each starts on the matrices the previous one left in L2.
  int run(GemmArgs& g) {
    g.reverse_batch = reverse ? 1 : 0;
    reverse = !reverse;
    return launch_gemm(g, stream);
  }

  GemmArgs base() const {
    GemmArgs g{};
    g.ab_dtype = kF16;
    g.batch = batch;
    g.round_dtype = -1;
    g.d_dtype = kF16;
    g.c_dtype = kF16;
    g.alpha = 1.0f;
    return g;
  }

  // G = X X^T (wide) or X^T X (tall), written to buf.g.
  int gram(const __half* x) {
    GemmArgs g = base();
    g.m = m;
    g.n = m;
    g.k = n;
    if (!tall) {
      g.a = {x, buf.xb, buf.ldx, 1};
      g.b = {x, buf.xb, 1, buf.ldx};
    } else {
      g.a = {x, buf.xb, 1, buf.ldx};
      g.b = {x, buf.xb, buf.ldx, 1};
    }
    g.d = buf.g;
    g.d_bstride = buf.mb;
    g.d_rstride = buf.ldm;
    g.symmetric = 1;
    g.upper_out = 1;
    return run(g);
  }

  // D = alpha A B + beta C over symmetric m x m operands (B read through its transpose).
  // Operands and outputs are stored as upper block triangles, except that
  // full_out writes D (and D2) whole: for a matrix whose next reader is an
  // X-product or a product that would otherwise switch operand layout.
  int sym(const __half* A, const __half* B, const __half* C, float alpha, float beta, __half* D, __half* D2,
          float gamma2, bool full_out = false) {
    GemmArgs g = base();
    g.m = m;
    g.n = m;
    g.k = m;
    g.a = {A, buf.mb, buf.ldm, 1};
    g.b = {B, buf.mb, 1, buf.ldm};
    g.c = (beta != 0.0f) ? C : nullptr;
    g.c_bstride = buf.mb;
    g.c_rstride = buf.ldm;
    g.alpha = alpha;
    g.beta = beta;
    g.d = D;
    g.d_bstride = buf.mb;
    g.d_rstride = buf.ldm;
    g.d2 = D2;
    g.d2_dtype = kF16;
    g.d2_bstride = buf.mb;
    g.d2_rstride = buf.ldm;
    g.gamma2 = gamma2;
    g.symmetric = 1;
    g.upper_out = full_out ? 0 : 1;
    g.a_upper = 1;
    g.b_upper = 1;
    return run(g);
  }

  // Iterations [it_begin, it_end) of the Gram recursion (newton_schulz.py:177-212),
  // starting from G in buf.g with no accumulated polynomial; Q ends in buf.q[qi].
  // The last iteration before a reset (or the last overall) skips the G update.
  // Iterations [it_begin, it_end) between two restarts; G is advanced after every
  // iteration but the segment's last (newton_schulz.py:177-212).
  int iterate(const double* coeffs, int it_begin, int it_end, int& qi) {
    bool have_q = false;
    for (int it = it_begin; it < it_end; ++it) {
      const float a = static_cast<float>(coeffs[3 * it + 0]);
      const float bq = static_cast<float>(coeffs[3 * it + 1]);
      const float c = static_cast<float>(coeffs[3 * it + 2]);
      int rc;
      // The segment's final Q is written whole: the X-product reading it then
      // loads every k-block K-major (switching operand layout inside a tile's
      // accumulation stalls the tensor pipe, about 0.9 us per tile on B200).
      const bool last = it + 1 == it_end;
      if (!have_q) {
        // P = c G^2 + b G, and Q = P + a I as a fused second output.
        rc = sym(buf.g, buf.g, buf.g, c, bq, buf.p, buf.q[qi], a, last);
        if (rc != GNS_OK) return rc;
        have_q = true;
      } else {
        rc = sym(buf.g, buf.g, buf.g, c, bq, buf.p, nullptr, 0.0f);
        if (rc != GNS_OK) return rc;
        rc = sym(buf.q[qi], buf.p, buf.q[qi], 1.0f, a, buf.q[qi ^ 1], nullptr, 0.0f, last);
        if (rc != GNS_OK) return rc;
        qi ^= 1;
      }
      if (it + 1 < it_end) {
        rc = sym(buf.g, buf.p, buf.g, 1.0f, a, buf.gp, nullptr, 0.0f);
        if (rc != GNS_OK) return rc;
        rc = sym(buf.p, buf.gp, buf.gp, 1.0f, a, buf.g, nullptr, 0.0f);
        if (rc != GNS_OK) return rc;
      }
    }
    return GNS_OK;
  }

  // Y = Q X (+ beta X) for wide, X Q (+ beta X) for tall; Y written with the given
  // layout/dtype. q_upper: Q is stored as its upper block triangle (else whole).
  int xproduct(const __half* Q, const __half* X, float beta, void* Y, int y_dtype, int64_t y_bstride,
               int64_t y_rstride, int round_dtype, bool q_upper) {
    GemmArgs g = base();
    if (!tall) {
      g.m = m;
      g.n = n;
      g.k = m;
      g.a = {Q, buf.mb, buf.ldm, 1};
      g.b = {X, buf.xb, buf.ldx, 1};
      g.a_upper = q_upper ? 1 : 0;
    } else {
      g.m = n;
      g.n = m;
      g.k = m;
      g.a = {X, buf.xb, buf.ldx, 1};
      g.b = {Q, buf.mb, 1, buf.ldm};
      g.b_upper = q_upper ? 1 : 0;
    }
    g.c = (beta != 0.0f) ? X : nullptr;
    g.c_bstride = buf.xb;
    g.c_rstride = buf.ldx;
    g.beta = beta;
    g.d = Y;
    g.d_dtype = y_dtype;
    g.d_bstride = y_bstride;
    g.d_rstride = y_rstride;
    g.round_dtype = round_dtype;
    return run(g);
  }
};

int check_chain_args(int x_dtype, int64_t batch, int64_t rows, int64_t cols, const void* x, void* out, int out_dtype,
                     const double* coeffs, int n_iters) {
  if (x_dtype < 0 || x_dtype > 2 || out_dtype < 0 || out_dtype > 2) return fail(GNS_ERR_ARGUMENT, "bad dtype");
  if (batch < 0 || rows < 0 || cols < 0) return fail(GNS_ERR_ARGUMENT, "negative dimension");
  if (n_iters < 0 || n_iters > 32) return fail(GNS_ERR_ARGUMENT, "n_iters must be in [0, 32]");
  if (n_iters > 0 && coeffs == nullptr) return fail(GNS_ERR_ARGUMENT, "null coefficients");
  if (batch > 0 && rows > 0 && cols > 0 && (x == nullptr || out == nullptr)) return fail(GNS_ERR_ARGUMENT, "null matrix");
  return GNS_OK;
}

// Gram-space-only workspace (G, P, GP, Q0, Q1) for gns_gram_iterations.
template <class Alloc>
void layout_gram_space(Alloc& al, ChainBuffers* cb, int64_t batch, int64_t m) {
  const int64_t ldm = round_up(m, 8), mb = m * ldm;
  const size_t mbytes = static_cast<size_t>(batch * mb) * 2;
  void* p[5];
  for (int i = 0; i < 5; ++i) {
    if constexpr (std::is_same<Alloc, Carver>::value) {
      p[i] = al.take(mbytes);
    } else {
      al.take(mbytes);
      p[i] = nullptr;
    }
  }
  if (cb) {
    cb->g = static_cast<__half*>(p[0]);
    cb->p = static_cast<__half*>(p[1]);
    cb->gp = static_cast<__half*>(p[2]);
    cb->q[0] = static_cast<__half*>(p[3]);
    cb->q[1] = static_cast<__half*>(p[4]);
    cb->ldm = ldm;
    cb->mb = mb;
  }
}

int launch_cast_square(const void* src, int src_f32, int src_upper, int64_t s_bstride, int64_t s_ld, __half* dst,
                       int64_t d_bstride, int64_t d_ld, int64_t batch, int64_t m, cudaStream_t stream) {
  const int64_t n = batch * m * m;
  int blocks = static_cast<int>((n + 255) / 256);
  if (blocks > 8 * device_sm_count()) blocks = 8 * device_sm_count();
  cast_square_to_half_kernel<<<blocks, 256, 0, stream>>>(src, src_f32, src_upper, s_bstride, s_ld, dst, d_bstride, d_ld,
                                                         batch, m);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GNS_OK : cuda_fail(e, "cast kernel");
}

int setup_chain(Chain& ch, int64_t batch, int64_t rows, int64_t cols, bool gram, void* workspace,
                size_t workspace_bytes, cudaStream_t stream) {
  ch.batch = batch;
  ch.rows = rows;
  ch.cols = cols;
  ch.tall = rows > cols;
  ch.m = ch.tall ? cols : rows;
  ch.n = ch.tall ? rows : cols;
  ch.stream = stream;
  Carver cv(workspace, workspace_bytes);
  layout_chain(cv, &ch.buf, batch, rows, cols, gram);
  if (cv.overflow) return fail(GNS_ERR_WORKSPACE, "Newton-Schulz workspace too small");
  return GNS_OK;
}

int cast_out(const Chain& ch, const __half* x, void* out, int out_dtype, int64_t obs, int64_t ors) {
  const int64_t nrows = ch.batch * ch.rows;
  const int64_t cap = 16 * static_cast<int64_t>(device_sm_count());
  const int blocks = static_cast<int>(nrows < cap ? nrows : cap);
  const int es = dtype_size(out_dtype);
  const int out_vec = (reinterpret_cast<uintptr_t>(out) % 16 == 0) && ((ors * es) % 16 == 0) &&
                      (ch.batch == 1 || (obs * es) % 16 == 0);
  cast_from_half_kernel<<<blocks, 256, 0, ch.stream>>>(x, ch.buf.ldx, ch.batch, ch.rows, ch.cols, out, out_dtype, obs,
                                                        ors, out_vec);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "cast kernel");
  return GNS_OK;
}

}  // namespace
}  // namespace gns

using namespace gns;

// Scratch of gns_frobenius_normalize_noalloc. Every GPU that loads this library
// holds these 64 KiB until the process exits. In host code the name is only a
// stand-in for the device array: kernels get the address that
// cudaGetSymbolAddress returns for the current device (noalloc_scratch_address).
static __device__ __align__(256) unsigned char g_noalloc_norm_scratch[64 * 1024];

namespace {

constexpr size_t kNoAllocScratchBytes = sizeof(g_noalloc_norm_scratch);
// Largest batch one allocation-free call accepts. The scratch holds one partial
// sum per (matrix, row slice) plus one arrival counter per matrix; a batch of at
// least four matrices per SM uses one slice per matrix, so 8192 matrices need
// 32 KiB + 32 KiB, and smaller batches need far less.
constexpr int64_t kNoAllocMaxBatch = 8192;

// Bytes of scratch one normalisation call uses: the same carve as launch_normalize.
size_t noalloc_scratch_need(int64_t batch, int64_t rows) {
  const int parts = norm_parts(batch, rows);
  const size_t partial_bytes = static_cast<size_t>(batch * parts) * sizeof(float);
  return ((partial_bytes + 255) & ~size_t(255)) + static_cast<size_t>(batch) * sizeof(unsigned int);
}

// Device address of the scratch on the current device. Host code cannot use the
// array's name as a device pointer, so every call asks the runtime (a host-side
// lookup that allocates nothing; the first one on a device also loads the module).
int noalloc_scratch_address(void** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_norm_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(normalize scratch)");
  *out = p;
  return GNS_OK;
}

}  // namespace

extern "C" {

size_t gns_normalize_workspace_size(int64_t batch, int64_t rows, int64_t cols) {
  return normalize_workspace_bytes(batch, rows, cols);
}

int gns_frobenius_normalize(int x_dtype, int64_t batch, int64_t rows, int64_t cols, const void* x, int64_t x_bstride,
                            int64_t x_rstride, void* out_f16, int64_t out_ld, float eps, void* workspace,
                            size_t workspace_bytes, gns_stream_t stream) {
  clear_error();
  if (batch > 0 && rows > 0 && cols > 0) {
    int rc = check_device();
    if (rc != GNS_OK) return rc;
  }
  return launch_normalize(x_dtype, batch, rows, cols, x, x_bstride, x_rstride, out_f16, out_ld, eps, workspace,
                          workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

// Allocation-free normalisation. Some callers cannot allocate device memory at
// the moment they normalise: code that must not call cudaMalloc (for example
// while another component owns every allocation through its own pool, or where
// an allocation could block or fail mid-step), or hosts that hand the library
// inputs and outputs but no workspace. This entry point therefore keeps its
// scratch (per-slice partial sums and per-matrix arrival counters) in the
// file-scope array g_noalloc_norm_scratch instead of a caller workspace.
int gns_frobenius_normalize_noalloc(int x_dtype, int64_t batch, int64_t rows, int64_t cols, const void* x,
                                    int64_t x_bstride, int64_t x_rstride, void* out_f16, int64_t out_ld, float eps,
                                    gns_stream_t stream) {
  clear_error();
  if (batch <= 0 || rows <= 0 || cols <= 0) {
    return launch_normalize(x_dtype, batch, rows, cols, x, x_bstride, x_rstride, out_f16, out_ld, eps, nullptr, 0,
                            reinterpret_cast<cudaStream_t>(stream));
  }
  int rc = check_device();
  if (rc != GNS_OK) return rc;
  if (batch > kNoAllocMaxBatch) {
    return fail(GNS_ERR_UNSUPPORTED, "gns_frobenius_normalize_noalloc: batch " + std::to_string(batch) +
                                         " exceeds the 8192 matrices its static scratch serves; use "
                                         "gns_frobenius_normalize with a workspace");
  }
  const size_t need = noalloc_scratch_need(batch, rows);
  if (need > kNoAllocScratchBytes) {
    return fail(GNS_ERR_UNSUPPORTED, "gns_frobenius_normalize_noalloc: this call needs " + std::to_string(need) +
                                         " bytes of scratch but the static scratch holds " +
                                         std::to_string(kNoAllocScratchBytes) + "; use gns_frobenius_normalize");
  }
  void* scratch = nullptr;
  rc = noalloc_scratch_address(&scratch);
  if (rc != GNS_OK) return rc;
  // launch_normalize zeroes the arrival counters (cudaMemsetAsync, no allocation)
  // before its kernel, so the previous call's leftovers never leak into this one.
  return launch_normalize(x_dtype, batch, rows, cols, x, x_bstride, x_rstride, out_f16, out_ld, eps, scratch,
                          kNoAllocScratchBytes, reinterpret_cast<cudaStream_t>(stream));
}

int gns_set_wait_limit_ns(unsigned long long limit_ns, unsigned long long* previous) {
  clear_error();
  if (limit_ns < 1000000ull || limit_ns > 10000000000ull)
    return fail(GNS_ERR_ARGUMENT, "wait limit must be between 1 ms and 10 s");
  const unsigned long long old = g_norm_wait_limit_ns.exchange(limit_ns);
  if (previous != nullptr) *previous = old;
  return GNS_OK;
}

int gns_selftest_normalize_timeout(int64_t batch, int64_t rows, int64_t cols, const float* x, void* out_f16,
                                   void* workspace, size_t workspace_bytes, gns_stream_t stream) {
  clear_error();
  if (batch <= 0 || rows <= 0 || cols <= 0) return fail(GNS_ERR_ARGUMENT, "empty self-test input");
  if (batch > 64 || rows * cols > (int64_t(1) << 20)) return fail(GNS_ERR_ARGUMENT, "self-test input too large");
  int rc = check_device();
  if (rc != GNS_OK) return rc;
  // One arrival more than the slices launched: nothing ever supplies it, so every
  // slice's bounded wait runs out after the current limit.
  return launch_normalize(GNS_F32, batch, rows, cols, x, rows * cols, cols, out_f16, cols, 1e-7f, workspace,
                          workspace_bytes, reinterpret_cast<cudaStream_t>(stream), 1u);
}

size_t gns_newton_schulz_workspace_size(int64_t batch, int64_t rows, int64_t cols) {
  Sizer s;
  layout_chain(s, nullptr, batch, rows, cols, true);
  return s.used + 256;
}

int gns_gram_newton_schulz(int x_dtype, int64_t batch, int64_t rows, int64_t cols, const void* x, int64_t x_bstride,
                           int64_t x_rstride, void* out, int out_dtype, int64_t out_bstride, int64_t out_rstride,
                           const double* coeffs, int n_iters, uint32_t reset_mask, float eps, void* workspace,
                           size_t workspace_bytes, gns_stream_t stream) {
  clear_error();
  int rc = check_chain_args(x_dtype, batch, rows, cols, x, out, out_dtype, coeffs, n_iters);
  if (rc != GNS_OK) return rc;
  if (n_iters == 0) return fail(GNS_ERR_ARGUMENT, "Gram Newton--Schulz requires coefficients");
  if (batch == 0 || rows == 0 || cols == 0) return GNS_OK;
  rc = check_device();
  if (rc != GNS_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  Chain ch;
  rc = setup_chain(ch, batch, rows, cols, true, workspace, workspace_bytes, st);
  if (rc != GNS_OK) return rc;
  ChainBuffers& B = ch.buf;

#define GNS_TRY(expr)        \
  do {                       \
    int _rc = (expr);        \
    if (_rc != GNS_OK) return _rc; \
  } while (0)

  GNS_TRY(launch_normalize(x_dtype, batch, rows, cols, x, x_bstride, x_rstride, B.x[0], B.ldx, eps, B.norm_ws,
                           B.norm_ws_bytes, st));
  if (small_chain_applies(batch, rows, cols))
    return launch_small_gram_chain(batch, rows, cols, B.x[0], B.x[1], B.ldx, B.xb, out, out_dtype, out_bstride,
                                   out_rstride, coeffs, n_iters, reset_mask, st);
  int xi = 0;
  GNS_TRY(ch.gram(B.x[xi]));
  int qi = 0;
  // Segments between restarts: at a reset iteration X <- Q X and G is rebuilt
  // (newton_schulz.py:164-175); resets at iteration 0 have no effect.
  int segment_begin = 0;
  for (int it = 1; it <= n_iters; ++it) {
    if (it < n_iters && !((reset_mask >> it) & 1u)) continue;
    GNS_TRY(ch.iterate(coeffs, segment_begin, it, qi));
    if (it < n_iters) {
      GNS_TRY(ch.xproduct(B.q[qi], B.x[xi], 0.0f, B.x[xi ^ 1], kF16, B.xb, B.ldx, -1, false));
      xi ^= 1;
      GNS_TRY(ch.gram(B.x[xi]));
    }
    segment_begin = it;
  }
  GNS_TRY(ch.xproduct(B.q[qi], B.x[xi], 0.0f, out, out_dtype, out_bstride, out_rstride, kF16, false));
  return GNS_OK;
}

int gns_standard_newton_schulz(int x_dtype, int64_t batch, int64_t rows, int64_t cols, const void* x,
                               int64_t x_bstride, int64_t x_rstride, void* out, int out_dtype, int64_t out_bstride,
                               int64_t out_rstride, const double* coeffs, int n_iters, float eps, void* workspace,
                               size_t workspace_bytes, gns_stream_t stream) {
  clear_error();
  int rc = check_chain_args(x_dtype, batch, rows, cols, x, out, out_dtype, coeffs, n_iters);
  if (rc != GNS_OK) return rc;
  if (batch == 0 || rows == 0 || cols == 0) return GNS_OK;
  rc = check_device();
  if (rc != GNS_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  Chain ch;
  rc = setup_chain(ch, batch, rows, cols, false, workspace, workspace_bytes, st);
  if (rc != GNS_OK) return rc;
  ChainBuffers& B = ch.buf;
  GNS_TRY(launch_normalize(x_dtype, batch, rows, cols, x, x_bstride, x_rstride, B.x[0], B.ldx, eps, B.norm_ws,
                           B.norm_ws_bytes, st));
  if (n_iters == 0) return cast_out(ch, B.x[0], out, out_dtype, out_bstride, out_rstride);
  if (small_square_applies(batch, rows, cols))
    return launch_small_standard_chain(batch, rows, B.x[0], B.ldx, B.xb, out, out_dtype, out_bstride, out_rstride,
                                       coeffs, n_iters, st);
  int xi = 0;
  for (int it = 0; it < n_iters; ++it) {
    const float a = static_cast<float>(coeffs[3 * it + 0]);
    const float bq = static_cast<float>(coeffs[3 * it + 1]);
    const float c = static_cast<float>(coeffs[3 * it + 2]);
    GNS_TRY(ch.gram(B.x[xi]));
    // P is read only by the X-product that follows: written whole (see iterate()).
    GNS_TRY(ch.sym(B.g, B.g, B.g, c, bq, B.p, nullptr, 0.0f, true));
    if (it == n_iters - 1 && out_dtype == kF16) {
      GNS_TRY(ch.xproduct(B.p, B.x[xi], a, out, out_dtype, out_bstride, out_rstride, -1, false));
    } else if (it == n_iters - 1) {
      // The accumulator X is fp16, so the last product lands in fp16 and is cast.
      GNS_TRY(ch.xproduct(B.p, B.x[xi], a, B.x[xi ^ 1], kF16, B.xb, B.ldx, -1, false));
      return cast_out(ch, B.x[xi ^ 1], out, out_dtype, out_bstride, out_rstride);
    } else {
      GNS_TRY(ch.xproduct(B.p, B.x[xi], a, B.x[xi ^ 1], kF16, B.xb, B.ldx, -1, false));
      xi ^= 1;
    }
  }
  return GNS_OK;
#undef GNS_TRY
}

// ------------------------------------------------ pieces of a sharded chain
int gns_frobenius_sumsq(int x_dtype, int64_t batch, int64_t rows, int64_t cols, const void* x, int64_t x_bstride,
                        int64_t x_rstride, float* sumsq_out, void* workspace, size_t workspace_bytes,
                        gns_stream_t stream) {
  clear_error();
  if (x_dtype < 0 || x_dtype > 2) return fail(GNS_ERR_ARGUMENT, "bad input dtype");
  if (batch < 0 || rows < 0 || cols < 0) return fail(GNS_ERR_ARGUMENT, "negative dimension");
  if (batch == 0) return GNS_OK;
  if (sumsq_out == nullptr) return fail(GNS_ERR_ARGUMENT, "null output");
  if (batch > 65535) return fail(GNS_ERR_UNSUPPORTED, "batch above 65535");
  int rc = check_device();
  if (rc != GNS_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (rows == 0 || cols == 0) {
    cudaError_t e = cudaMemsetAsync(sumsq_out, 0, static_cast<size_t>(batch) * sizeof(float), st);
    return e == cudaSuccess ? GNS_OK : cuda_fail(e, "zero sums");
  }
  if (x == nullptr) return fail(GNS_ERR_ARGUMENT, "null matrix");
  const int parts = norm_parts(batch, rows);
  const int64_t rpp = (rows + parts - 1) / parts;
  if (rpp * ((cols + 7) / 8) >= (int64_t(1) << 31)) return fail(GNS_ERR_UNSUPPORTED, "matrix slice too large");
  const int used = static_cast<int>((rows + rpp - 1) / rpp);
  if (workspace == nullptr || workspace_bytes < static_cast<size_t>(batch * used) * sizeof(float))
    return fail(GNS_ERR_WORKSPACE, "sum-of-squares workspace too small");
  const int64_t es = dtype_size(x_dtype);
  const int vec = (cols % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((x_rstride * es) % 16 == 0) &&
                  (batch == 1 || (x_bstride * es) % 16 == 0);
  float* partial = static_cast<float*>(workspace);
  sumsq_slices_kernel<<<dim3(used, static_cast<unsigned>(batch)), kNormThreads, 0, st>>>(
      x, x_dtype, rows, cols, x_bstride, x_rstride, rpp, vec, partial);
  sumsq_reduce_kernel<<<static_cast<unsigned>(batch), kNormThreads, 0, st>>>(partial, used, sumsq_out);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GNS_OK : cuda_fail(e, "sum-of-squares kernels");
}

int gns_frobenius_scale(int x_dtype, int64_t batch, int64_t rows, int64_t cols, const void* x, int64_t x_bstride,
                        int64_t x_rstride, const float* sumsq, float eps, void* out_f16, int64_t out_ld,
                        gns_stream_t stream) {
  clear_error();
  if (x_dtype < 0 || x_dtype > 2) return fail(GNS_ERR_ARGUMENT, "bad input dtype");
  if (batch < 0 || rows < 0 || cols < 0) return fail(GNS_ERR_ARGUMENT, "negative dimension");
  if (out_ld < cols) return fail(GNS_ERR_ARGUMENT, "out_ld < cols");
  if (batch == 0 || rows == 0 || cols == 0) return GNS_OK;
  if (x == nullptr || sumsq == nullptr || out_f16 == nullptr) return fail(GNS_ERR_ARGUMENT, "null tensor");
  if (batch > 65535) return fail(GNS_ERR_UNSUPPORTED, "batch above 65535");
  int rc = check_device();
  if (rc != GNS_OK) return rc;
  const int parts = norm_parts(batch, rows);
  const int64_t rpp = (rows + parts - 1) / parts;
  if (rpp * ((cols + 7) / 8) >= (int64_t(1) << 31)) return fail(GNS_ERR_UNSUPPORTED, "matrix slice too large");
  const int used = static_cast<int>((rows + rpp - 1) / rpp);
  const int64_t es = dtype_size(x_dtype);
  const int vec = (cols % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((x_rstride * es) % 16 == 0) &&
                  (batch == 1 || (x_bstride * es) % 16 == 0) && (reinterpret_cast<uintptr_t>(out_f16) % 16 == 0) &&
                  (out_ld % 8 == 0);
  scale_with_sumsq_kernel<<<dim3(used, static_cast<unsigned>(batch)), kNormThreads, 0,
                            reinterpret_cast<cudaStream_t>(stream)>>>(x, x_dtype, rows, cols, x_bstride, x_rstride,
                                                                      rpp, vec, sumsq, eps,
                                                                      static_cast<__half*>(out_f16), out_ld);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GNS_OK : cuda_fail(e, "scale kernel");
}

size_t gns_gram_iterations_workspace_size(int64_t batch, int64_t m) {
  Sizer s;
  layout_gram_space(s, nullptr, batch, m);
  return s.used + 256;
}

int gns_gram_iterations(int64_t batch, int64_t m, const void* gram, int gram_f32, int64_t g_bstride, int64_t g_rstride,
                        const double* coeffs, int n_iters, int it_begin, int it_end, void* q_out,
                        int64_t q_bstride, int64_t q_rstride, void* workspace, size_t workspace_bytes,
                        gns_stream_t stream) {
  clear_error();
  if (batch < 0 || m < 0) return fail(GNS_ERR_ARGUMENT, "negative dimension");
  if (n_iters < 1 || n_iters > 32 || coeffs == nullptr) return fail(GNS_ERR_ARGUMENT, "need 1..32 coefficient triples");
  if (it_begin < 0 || it_begin >= it_end || it_end > n_iters) return fail(GNS_ERR_ARGUMENT, "bad iteration range");
  if (batch == 0 || m == 0) return GNS_OK;
  if (gram == nullptr || q_out == nullptr) return fail(GNS_ERR_ARGUMENT, "null tensor");
  int rc = check_device();
  if (rc != GNS_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  Chain ch;
  ch.batch = batch;
  ch.rows = ch.cols = ch.m = ch.n = m;
  ch.tall = false;
  ch.stream = st;
  Carver cv(workspace, workspace_bytes);
  layout_gram_space(cv, &ch.buf, batch, m);
  if (cv.overflow) return fail(GNS_ERR_WORKSPACE, "Gram iteration workspace too small");
  ChainBuffers& B = ch.buf;
  rc = launch_cast_square(gram, gram_f32 ? 1 : 0, 0, g_bstride, g_rstride, B.g, B.mb, B.ldm, batch, m, st);
  if (rc != GNS_OK) return rc;
  int qi = 0;
  rc = ch.iterate(coeffs, it_begin, it_end, qi);
  if (rc != GNS_OK) return rc;
  // Q is kept as its upper block triangle inside the chain; the caller gets it whole.
  return launch_cast_square(B.q[qi], 0, 1, B.mb, B.ldm, static_cast<__half*>(q_out), q_bstride, q_rstride, batch, m,
                            st);
}

}  // extern "C"
