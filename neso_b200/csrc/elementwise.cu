// vector_add and scale (windows/kernels.py:7-22, tests/test_aot.py:17-28).
//
// HBM streaming kernels: 128-bit (float4) loads and stores with evict-first
// cache hints, one float4 per thread per iteration, grid-stride over 64 CTAs
// of 256 threads per SM (eight resident at a time): measured on B200 at
// n = 2^28, scale 6126 -> 6572 GB/s and add 6337 -> 6771 GB/s against four
// float4 per thread over eight CTAs per SM (more CTAs in turn beat deeper
// unrolling: 16 x 2: 6249 / 6627, 32 x 2: 6394 / 6708; one CTA per 1024
// elements, no grid stride: 4781 / 6107). Arithmetic is one IEEE fp32 add or
// multiply per element (no contraction is possible), so results are
// bit-identical to torch's `x + y` and `x * a`. The reference's BLOCK_SIZE and
// grid only describe the reference launch; they are validated, not used.
#include "runtime.h"

namespace neso {
namespace {

constexpr int kThreads = 256;
constexpr int kCtasPerSm = 64;

template <bool kAdd>
__global__ void __launch_bounds__(kThreads) ew_vec4_kernel(const float4* __restrict__ x, const float4* __restrict__ y,
                                                           float4* __restrict__ out, float factor, int64_t n4) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  for (; i < n4; i += stride) {
    float4 a = __ldcs(x + i);
    float4 r;
    if (kAdd) {
      float4 b = __ldcs(y + i);
      r = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
    } else {
      r = make_float4(a.x * factor, a.y * factor, a.z * factor, a.w * factor);
    }
    __stcs(out + i, r);
  }
}

// Scalar path: the <4-element tail of the vector path, or whole arrays whose
// pointers are not 16-byte aligned.
template <bool kAdd>
__global__ void __launch_bounds__(kThreads) ew_scalar_kernel(const float* __restrict__ x, const float* __restrict__ y,
                                                             float* __restrict__ out, float factor, int64_t begin,
                                                             int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = begin + static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride) {
    out[i] = kAdd ? (x[i] + y[i]) : (x[i] * factor);
  }
}

int validate_grid(int32_t n, int32_t block, uint32_t gx, uint32_t gy, uint32_t gz) {
  if (n < 0) return fail(NESO_ERR_INVALID_ARG, "n_elements must be >= 0 (got %d)", n);
  if (block < 1 || block > (1 << 20) || (block & (block - 1)) != 0) {
    return fail(NESO_ERR_INVALID_ARG, "BLOCK_SIZE must be a power of two (got %d)", block);
  }
  const uint32_t want = static_cast<uint32_t>((static_cast<int64_t>(n) + block - 1) / block);
  if (gx != want || gy != 1 || gz != 1) {
    return fail(NESO_ERR_GRID, "grid (%u,%u,%u) != (cdiv(%d,%d)=%u,1,1)", gx, gy, gz, n, block, want);
  }
  return NESO_OK;
}

template <bool kAdd>
int launch_ew(const float* x, const float* y, float* out, float factor, int64_t n, cudaStream_t stream) {
  if (n == 0) return ok();
  if (x == nullptr || out == nullptr || (kAdd && y == nullptr)) return fail(NESO_ERR_INVALID_ARG, "null pointer");
  const int sms = sm_count();
  const int max_blocks = sms * kCtasPerSm;
  const bool vec = aligned16(x) && aligned16(out) && (!kAdd || aligned16(y));
  if (vec) {
    const int64_t n4 = n / 4;
    if (n4 > 0) {
      int64_t want = (n4 + kThreads - 1) / kThreads;
      int blocks = static_cast<int>(want < max_blocks ? want : max_blocks);
      ew_vec4_kernel<kAdd><<<blocks, kThreads, 0, stream>>>(reinterpret_cast<const float4*>(x),
                                                            reinterpret_cast<const float4*>(y),
                                                            reinterpret_cast<float4*>(out), factor, n4);
    }
    if (n4 * 4 < n) ew_scalar_kernel<kAdd><<<1, kThreads, 0, stream>>>(x, y, out, factor, n4 * 4, n);
  } else {
    int64_t want = (n + kThreads - 1) / kThreads;
    int blocks = static_cast<int>(want < max_blocks ? want : max_blocks);
    ew_scalar_kernel<kAdd><<<blocks, kThreads, 0, stream>>>(x, y, out, factor, 0, n);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, kAdd ? "vector_add launch" : "scale launch");
  return ok();
}

}  // namespace
}  // namespace neso

using namespace neso;

extern "C" {

int neso_vector_add(const float* x, const float* y, float* output, int32_t n_elements, int32_t BLOCK_SIZE,
                    uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream) {
  int rc = validate_grid(n_elements, BLOCK_SIZE, grid_x, grid_y, grid_z);
  if (rc != NESO_OK) return rc;
  return launch_ew<true>(x, y, output, 0.f, n_elements, as_stream(stream));
}

int neso_add_kernel(const float* x_ptr, const float* y_ptr, float* z_ptr, int32_t n_elements, int32_t BLOCK_SIZE,
                    uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream) {
  return neso_vector_add(x_ptr, y_ptr, z_ptr, n_elements, BLOCK_SIZE, grid_x, grid_y, grid_z, stream);
}

int neso_scale(const float* x, float* output, float factor, int32_t n_elements, int32_t BLOCK_SIZE, uint32_t grid_x,
               uint32_t grid_y, uint32_t grid_z, neso_stream_t stream) {
  int rc = validate_grid(n_elements, BLOCK_SIZE, grid_x, grid_y, grid_z);
  if (rc != NESO_OK) return rc;
  return launch_ew<false>(x, nullptr, output, factor, n_elements, as_stream(stream));
}

}  // extern "C"
