// Host-side plumbing shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace gns {

// Records `msg` as this thread's last error and returns `code`.
int fail(int code, const std::string& msg);
// Wraps a CUDA runtime error.
int cuda_fail(cudaError_t err, const char* what);
// Clears the thread's last error.
void clear_error();

// Current device's SM count (cached per device).
int device_sm_count();
// Returns GNS_OK when the current device is an sm_100 part.
int check_device();

// Round up to a multiple.
inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// Workspace carving helper: 256-byte aligned bump allocator over a caller buffer.
struct Carver {
  uint8_t* base;
  size_t cap;
  size_t used = 0;
  bool overflow = false;
  Carver(void* p, size_t bytes) : base(static_cast<uint8_t*>(p)), cap(bytes) {}
  void* take(size_t bytes) {
    size_t off = (used + 255) & ~size_t(255);
    used = off + bytes;
    if (used > cap || base == nullptr) {
      overflow = true;
      return nullptr;
    }
    return base + off;
  }
};

// Size computation counterpart of Carver.
struct Sizer {
  size_t used = 0;
  void take(size_t bytes) { used = ((used + 255) & ~size_t(255)) + bytes; }
};

// One matrix operand as the GEMM sees it: logical [batch, rows, cols] with strides.
struct Operand {
  const void* ptr;
  int64_t bstride, rstride, cstride;
};

struct GemmArgs {
  int ab_dtype;
  int64_t batch, m, n, k;
  Operand a, b;  // A [m, k], B [k, n]
  const void* c;
  int c_dtype;
  int64_t c_bstride, c_rstride;
  void* d;
  int d_dtype;
  int64_t d_bstride, d_rstride;
  int round_dtype;  // -1 or dtype to round through before the D cast
  void* d2;         // optional second output (symmetric chains: Q = P + gamma2 * I)
  int d2_dtype;
  int64_t d2_bstride, d2_rstride;
  float gamma2;
  float alpha, beta;
  int symmetric;
  int reverse_batch;  // traverse the batch last-to-first
  // Upper block-triangle storage of symmetric m x m matrices (256 x 256 blocks,
  // column block >= row block), used inside the chains: upper_out writes a
  // symmetric product that way (no mirrored lower blocks); a_upper / b_upper
  // mark a square K-major operand stored that way (lower tiles read transposed).
  int upper_out, a_upper, b_upper;
};

// Validates, builds the tensor maps and launches the tcgen05 GEMM.
int launch_gemm(const GemmArgs& g, cudaStream_t stream);

// Status word of the normalisation kernel (0 = ok); optionally cleared.
int normalize_status(int* status, int clear);

// Normalisation: out = fp16(x / (||x||_F + eps)) per matrix.
size_t normalize_workspace_bytes(int64_t batch, int64_t rows, int64_t cols);
// extra_arrivals > 0 makes every slice wait for arrivals that never come, so the
// bounded wait runs out (gns_selftest_normalize_timeout); 0 everywhere else.
int launch_normalize(int x_dtype, int64_t batch, int64_t rows, int64_t cols, const void* x,
                     int64_t x_bstride, int64_t x_rstride, void* out, int64_t out_ld, float eps,
                     void* workspace, size_t workspace_bytes, cudaStream_t stream,
                     unsigned int extra_arrivals = 0);

// Encodes a 3-D fp16 tensor map [batch][outer][inner] with a {64, box_outer, 1}
// box and 128-byte swizzle (the GEMM's operand maps).
int encode_f16_tiles(CUtensorMap* map, const void* ptr, int64_t inner, int64_t outer, int64_t batch,
                     int64_t outer_stride, int64_t batch_stride, int box_outer);

// Fused single-kernel Gram Newton-Schulz chain for matrices whose short side is
// at most 128 (small_chain.cu). x0 holds the normalised fp16 X and x1 is the
// reset buffer, both [batch][rows][ldx].
bool small_chain_applies(int64_t batch, int64_t rows, int64_t cols);
int launch_small_gram_chain(int64_t batch, int64_t rows, int64_t cols, __half* x0, __half* x1, int64_t ldx,
                            int64_t xb, void* out, int out_dtype, int64_t out_bstride, int64_t out_rstride,
                            const double* coeffs, int n_iters, uint32_t reset_mask, cudaStream_t stream);
int small_chain_status(int* status, int clear);
// The same kernel for the standard chain of square matrices with side <= 128.
bool small_square_applies(int64_t batch, int64_t rows, int64_t cols);
int launch_small_standard_chain(int64_t batch, int64_t m, __half* x0, int64_t ldx, int64_t xb, void* out,
                                int out_dtype, int64_t out_bstride, int64_t out_rstride, const double* coeffs,
                                int n_iters, cudaStream_t stream);

}  // namespace gns
