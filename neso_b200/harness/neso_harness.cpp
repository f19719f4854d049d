// neso_harness — native correctness and performance harness on the C ABI.
//
// Re-hosts the protocol of the reference's native harnesses
// (macos/harness.rs:201-365, windows/harness.rs:118-308) on CUDA:
//   test   vector_add on n = 65 537 (masked tail, BLOCK 256), scale with
//          factor -1.75, and the FA2 known answer (Q = K = 0: every O row is
//          the column mean of fp16(V), V_i = ((i % 17) - 8) * 0.125, N = 64,
//          d = 64, tolerance 2e-3). Elementwise results must be bit-exact.
//   bench  vector_add / scale over 16 Mi elements (GB/s = 12n / t, 8n / t)
//          and single-head FA2 d = 64 for N = 128 ... 2048 (GFLOP/s =
//          4 N^2 d / t): 10 warm-up launches, then the median of 50 (20 for
//          FA2) launches, each timed with CUDA events.
// Exit status is non-zero on any failure.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <vector>

#include "neso_b200.h"

namespace {

constexpr int kBlock = 256;   // macos/harness.rs:15
constexpr int kFa2BlockM = 16;
constexpr int kHeadDim = 64;

bool check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    std::fprintf(stderr, "FAIL %s: %s\n", what, cudaGetErrorString(e));
    return false;
  }
  return true;
}

bool check_neso(int rc, const char* what) {
  if (rc != NESO_OK) {
    std::fprintf(stderr, "FAIL %s: status %d: %s\n", what, rc, neso_last_error_string());
    return false;
  }
  return true;
}

unsigned groups(long n, int block) { return static_cast<unsigned>((n + block - 1) / block); }

template <class T>
struct DeviceBuf {
  T* p = nullptr;
  size_t n = 0;
  explicit DeviceBuf(size_t count) : n(count) {
    if (cudaMalloc(&p, count * sizeof(T)) != cudaSuccess) p = nullptr;
  }
  ~DeviceBuf() { cudaFree(p); }
  bool upload(const std::vector<T>& h) { return cudaMemcpy(p, h.data(), n * sizeof(T), cudaMemcpyHostToDevice) == cudaSuccess; }
  std::vector<T> download() const {
    std::vector<T> h(n);
    cudaMemcpy(h.data(), p, n * sizeof(T), cudaMemcpyDeviceToHost);
    return h;
  }
};

// macos/harness.rs:171-183
void fa2_values(int n, std::vector<float>& q, std::vector<float>& k, std::vector<float>& v) {
  const int count = n * kHeadDim;
  q.resize(count);
  k.resize(count);
  v.resize(count);
  for (int i = 0; i < count; ++i) {
    q[i] = static_cast<float>(i % 29 - 14) * 0.01f;
    k[i] = static_cast<float>(i % 31 - 15) * 0.01f;
    v[i] = static_cast<float>(i % 17 - 8) * 0.125f;
  }
}

std::vector<__half> to_half(const std::vector<float>& f) {
  std::vector<__half> h(f.size());
  for (size_t i = 0; i < f.size(); ++i) h[i] = __float2half_rn(f[i]);
  return h;
}

int fa2(const __half* q, const __half* k, const __half* v, float* o, int n, cudaStream_t s) {
  const float scale = 1.0f / std::sqrt(static_cast<float>(kHeadDim));
  return neso_flash_attention_fwd(q, k, v, o, n, kHeadDim, kHeadDim, scale, kHeadDim, n / kFa2BlockM, 1, 1, s);
}

int run_test() {
  bool ok = true;
  const int count = 65537;
  std::vector<float> x(count), y(count);
  for (int i = 0; i < count; ++i) {
    x[i] = (static_cast<float>(i) - 1000.0f) * 0.125f;
    y[i] = static_cast<float>(i % 97) * -0.25f;
  }
  DeviceBuf<float> xd(count), yd(count), od(count);
  if (!xd.p || !yd.p || !od.p || !xd.upload(x) || !yd.upload(y)) return check_cuda(cudaErrorMemoryAllocation, "setup"), 1;

  ok &= check_neso(neso_vector_add(xd.p, yd.p, od.p, count, kBlock, groups(count, kBlock), 1, 1, nullptr), "vector_add");
  ok &= check_cuda(cudaDeviceSynchronize(), "vector_add");
  {
    std::vector<float> out = od.download();
    size_t bad = 0;
    float e = 0;
    for (int i = 0; i < count; ++i) {
      const float want = x[i] + y[i];
      bad += std::memcmp(&out[i], &want, 4) != 0;
      e = std::max(e, std::fabs(out[i] - want));
    }
    if (bad == 0 && e <= 1e-6f) {
      std::printf("PASS vector_add (%d elements, masked tail, bit-exact)\n", count);
    } else {
      std::printf("FAIL vector_add: %zu elements differ, max error %g\n", bad, e);
      ok = false;
    }
  }

  const float factor = -1.75f;
  ok &= check_neso(neso_scale(xd.p, od.p, factor, count, kBlock, groups(count, kBlock), 1, 1, nullptr), "scale");
  ok &= check_cuda(cudaDeviceSynchronize(), "scale");
  {
    std::vector<float> out = od.download();
    size_t bad = 0;
    for (int i = 0; i < count; ++i) {
      const float want = x[i] * factor;
      bad += std::memcmp(&out[i], &want, 4) != 0;
    }
    if (bad == 0) {
      std::printf("PASS scale (%d elements, scalar argument, bit-exact)\n", count);
    } else {
      std::printf("FAIL scale: %zu elements differ\n", bad);
      ok = false;
    }
  }

  const int n = 64;
  std::vector<float> qf, kf, vf;
  fa2_values(n, qf, kf, vf);
  std::vector<float> zeros(n * kHeadDim, 0.0f);
  std::vector<__half> zh = to_half(zeros), vh = to_half(vf);
  DeviceBuf<__half> qd(n * kHeadDim), kd(n * kHeadDim), vd(n * kHeadDim);
  DeviceBuf<float> fo(n * kHeadDim);
  qd.upload(zh);
  kd.upload(zh);
  vd.upload(vh);
  ok &= check_neso(fa2(qd.p, kd.p, vd.p, fo.p, n, nullptr), "flash_attention_fwd");
  ok &= check_cuda(cudaDeviceSynchronize(), "flash_attention_fwd");
  {
    std::vector<float> out = fo.download();
    std::vector<float> mean(kHeadDim, 0.0f);
    for (int r = 0; r < n; ++r)
      for (int c = 0; c < kHeadDim; ++c) mean[c] += __half2float(vh[r * kHeadDim + c]);
    for (float& m : mean) m /= n;
    float e = 0;
    for (int r = 0; r < n; ++r)
      for (int c = 0; c < kHeadDim; ++c) e = std::max(e, std::fabs(out[r * kHeadDim + c] - mean[c]));
    if (e <= 2e-3f) {
      std::printf("PASS flash_attention_2 (f16, N=%d, d=%d, max error %.2e)\n", n, kHeadDim, e);
    } else {
      std::printf("FAIL flash_attention_2: max error %g\n", e);
      ok = false;
    }
  }
  int code = 0;
  ok &= check_neso(neso_device_status(0, &code, nullptr, nullptr, nullptr), "device status");
  return ok ? 0 : 1;
}

// macos/harness.rs:280-292: warm-ups, then the median of `iterations` samples.
double measure_ms(const std::function<int()>& launch, int iterations, bool* ok) {
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  for (int i = 0; i < 10; ++i) *ok &= launch() == NESO_OK;
  std::vector<float> samples;
  for (int i = 0; i < iterations; ++i) {
    cudaEventRecord(a);
    *ok &= launch() == NESO_OK;
    cudaEventRecord(b);
    cudaEventSynchronize(b);
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    samples.push_back(ms);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  std::sort(samples.begin(), samples.end());
  return samples[samples.size() / 2];
}

int run_bench() {
  bool ok = true;
  const int count = 16 * 1024 * 1024;
  DeviceBuf<float> xd(count), yd(count), od(count);
  xd.upload(std::vector<float>(count, 1.0f));
  yd.upload(std::vector<float>(count, 2.0f));
  const double add_ms = measure_ms(
      [&] { return neso_vector_add(xd.p, yd.p, od.p, count, kBlock, groups(count, kBlock), 1, 1, nullptr); }, 50, &ok);
  std::printf("vector_add  %8.3f ms  %8.2f GB/s\n", add_ms, count * 12.0 / (add_ms * 1e-3) / 1e9);
  const double scale_ms = measure_ms(
      [&] { return neso_scale(xd.p, od.p, 1.25f, count, kBlock, groups(count, kBlock), 1, 1, nullptr); }, 50, &ok);
  std::printf("scale       %8.3f ms  %8.2f GB/s\n", scale_ms, count * 8.0 / (scale_ms * 1e-3) / 1e9);

  const int nmax = 2048;
  std::vector<float> qf, kf, vf;
  fa2_values(nmax, qf, kf, vf);
  DeviceBuf<__half> qd(nmax * kHeadDim), kd(nmax * kHeadDim), vd(nmax * kHeadDim);
  DeviceBuf<float> fo(nmax * kHeadDim);
  qd.upload(to_half(qf));
  kd.upload(to_half(kf));
  vd.upload(to_half(vf));
  for (int n : {128, 256, 512, 1024, 2048}) {
    const double ms = measure_ms([&] { return fa2(qd.p, kd.p, vd.p, fo.p, n, nullptr); }, 20, &ok);
    const double flops = 4.0 * n * n * kHeadDim;
    std::printf("flash_attn2 f16 N=%4d d=%d  %8.3f ms  %8.2f GFLOP/s\n", n, kHeadDim, ms, flops / (ms * 1e-3) / 1e9);
  }
  ok &= check_cuda(cudaDeviceSynchronize(), "bench");
  return ok ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
  const char* mode = argc > 1 ? argv[1] : "";
  if (std::strcmp(mode, "test") == 0) return run_test();
  if (std::strcmp(mode, "bench") == 0) return run_bench();
  std::fprintf(stderr, "usage: neso_harness <test|bench>\n");
  return 2;
}
