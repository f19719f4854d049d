// Dequant-fused quantized matmul on sm_100a: W8A16 (per-output-channel fp16
// scale) and packed W4A16 (group 128, fp16 scale per group).
//
// Reference kernels: tests/test_quantized_matmul.py:67-167 (w8a16_matmul:
// load i8 -> sitofp -> f16 -> tt.dot, fp32 C), :181-283 (w8a16_scaled_matmul:
// per-channel scale in the fp32 epilogue, :250-260), :170-178 (W4A16 stored one
// value per byte = the W8A16 kernel with values in [-8, 7]). The packed int4
// group-128 variant has no reference kernel; its group semantics follow the
// grouped dequant of tests/test_advanced12.py:69-84.
//
// One persistent CTA per SM; per 64-deep K block ("stage"):
//   warp 0      TMA: raw weight tile (int8 [64 k][128 n] or packed int4
//               [32 byte-rows][128 n], 128-byte swizzled), the fp16
//               activation tile, and (int4) the group's fp16 scale row.
//   warps 4-7   dequantise raw -> fp16 directly into the MN-major 128-byte
//               swizzled layout tcgen05 reads; fence.proxy.async; arrive.
//                 int8: exact, (b ^ 0x80) | 0x6400 as fp16 is 1024 + b + 128.
//                 int4: q exact the same way, then w = q * s is split into
//                 w_hi = fp16(q * s) and w_lo = fma(q, s, -w_hi) (the exact
//                 rounding error), so the MMA sums q * s without rounding it.
//   warp 1      tcgen05.mma issuer (kind::f16, fp32 accumulator in TMEM,
//               double-buffered); int4 issues hi and lo MMAs per K step.
//   warps 8-11  epilogue: TMEM -> registers -> (int8: * f32(scale[n])) -> Y.
// Orientation: M >= 65 computes Y tiles [128 m x 128 n] with X as the A
// operand; M <= 64 swaps operands (A = dequantised W^T with M' = 128 output
// channels, B = X with N' = M rounded up to 16/32/64) so decode-sized batches
// still run on the tensor cores and the weight stream stays at HBM speed.
#include "runtime.h"

namespace neso {
namespace {

constexpr int kThreads = 384;
constexpr int kBK = 64;
constexpr int kTileN = 128;  // output channels per tile

enum QuantKind : int { kInt8 = 0, kInt4G128 = 1 };

template <int kQ, bool kSwap, int kNX>
struct QCfg {
  static constexpr int kXBytes = kNX * kBK * 2;                  // X tile [kNX rows][64 k] fp16
  static constexpr int kRawBytes = (kQ == kInt8) ? 64 * 128 : 32 * 128;
  static constexpr int kW16Bytes = kBK * kTileN * 2;             // 16 KB per fp16 copy
  static constexpr int kNumW16 = (kQ == kInt8) ? 1 : 2;          // int4: hi + lo
  static constexpr int kScaleBytes = (kQ == kInt8) ? 0 : 1024;   // 256 B used, padded for alignment
  static constexpr int kStageBytes = kXBytes + kRawBytes + kNumW16 * kW16Bytes + kScaleBytes;
  static constexpr int kStagesRaw = (220 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kAccCols = kSwap ? kNX : kTileN;          // accumulator columns per buffer
  static constexpr int kTmemCols = (2 * kAccCols <= 32) ? 32 : (2 * kAccCols <= 64) ? 64
                                   : (2 * kAccCols <= 128) ? 128 : 256;
  static constexpr int kTxBytes = kXBytes + kRawBytes + ((kQ == kInt8) ? 0 : 256);
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 512;
  // offsets within a stage (all 1024-aligned)
  static constexpr int kOffX = 0;
  static constexpr int kOffRaw = kXBytes;
  static constexpr int kOffW16 = kXBytes + kRawBytes;
  static constexpr int kOffScale = kOffW16 + kNumW16 * kW16Bytes;
  static_assert(kXBytes % 1024 == 0 && kRawBytes % 1024 == 0, "stage parts must stay 1024-aligned");
};

struct QArgs {
  float* Y;
  int64_t ldy;
  const __half* chan_scale;  // int8: per-channel scale [N] (nullable)
  int M, N, K;
  int num_m, num_n, num_k;
  DevStatus st;
};

// fp16 pair (lo = byte b0, hi = byte b1 of x) -> 0x6400 | byte, i.e. 1024 + byte.
__device__ __forceinline__ uint32_t bytes_to_h2(uint32_t x, uint32_t sel) {
  return __byte_perm(x, 0x64646464u, sel);
}

__device__ __forceinline__ __half2 u32_as_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }
__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Convert 16 int8 weights (one 16-byte raw unit) into two 16-byte fp16 units.
__device__ __forceinline__ void dequant_i8x16(uint4 raw, uint4& o0, uint4& o1) {
  const __half2 bias = __float2half2_rn(1152.f);  // 1024 + 128
  uint32_t w[4] = {raw.x ^ 0x80808080u, raw.y ^ 0x80808080u, raw.z ^ 0x80808080u, raw.w ^ 0x80808080u};
  uint32_t h[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    h[2 * i] = h2_as_u32(__hsub2(u32_as_h2(bytes_to_h2(w[i], 0x5140)), bias));
    h[2 * i + 1] = h2_as_u32(__hsub2(u32_as_h2(bytes_to_h2(w[i], 0x7362)), bias));
  }
  o0 = make_uint4(h[0], h[1], h[2], h[3]);
  o1 = make_uint4(h[4], h[5], h[6], h[7]);
}

template <int kQ, bool kSwap, int kNX>
__global__ void __launch_bounds__(kThreads, 1)
    wq_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmS, QArgs args) {
  using Cfg = QCfg<kQ, kSwap, kNX>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* load_full = bars;            // [S] TMA bytes landed
  uint64_t* conv_full = bars + S;        // [S] fp16 weights written (4 warps)
  uint64_t* stage_empty = bars + 2 * S;  // [S] MMAs done with the stage
  uint64_t* acc_full = bars + 3 * S;     // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2] (4 epilogue warps)
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* never_flag = abort_flag + 1;  // stays 0: drain waits ignore the abort

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int num_tiles = args.num_m * args.num_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&load_full[s], 1);
      mbar_init(&conv_full[s], 4);
      mbar_init(&stage_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    *never_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
    if (kQ == kInt4G128) tma_prefetch_desc(&tmS);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer --
    int it = 0;
    bool aborted = false;
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x) {
      const int mb = t % args.num_m;
      const int nb = t / args.num_m;
      for (int kb = 0; kb < args.num_k; ++kb, ++it) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (!mbar_wait(&stage_empty[s], ph ^ 1, abort_flag, args.st, 0x2100)) { aborted = true; break; }
        uint8_t* st = smem + s * Cfg::kStageBytes;
        mbar_arrive_expect_tx(&load_full[s], Cfg::kTxBytes);
        tma_load_2d(st + Cfg::kOffX, &tmX, &load_full[s], kb * kBK, kSwap ? 0 : mb * 128);
        if (kQ == kInt8) {
          tma_load_2d(st + Cfg::kOffRaw, &tmW, &load_full[s], nb * kTileN, kb * kBK);
        } else {
          tma_load_2d(st + Cfg::kOffRaw, &tmW, &load_full[s], nb * kTileN, kb * (kBK / 2));
          tma_load_2d(st + Cfg::kOffScale, &tmS, &load_full[s], nb * kTileN, (kb * kBK) / 128);
        }
      }
    }
    if (aborted) {
      DevStatus quiet = args.st;
      quiet.word = nullptr;
      for (int i = (it > S ? it - S : 0); i < it; ++i) mbar_wait(&load_full[i % S], (i / S) & 1, never_flag, quiet, 0);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------- MMA issuer --
    // normal: A = X [128 m x 64 k] K-major, B = W16 [64 k x 128 n] MN-major
    // swap:   A = W16 as [128 n x 64 k] MN-major, B = X [kNX m x 64 k] K-major
    constexpr uint32_t idesc = kSwap ? idesc_f16_f32(128, kNX, 1, 0) : idesc_f16_f32(128, kTileN, 0, 1);
    int it = 0, tc = 0;
    bool aborted = false;
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x, ++tc) {
      const int buf = tc & 1;
      const uint32_t use = tc >> 1;
      if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, abort_flag, args.st, 0x2200)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem + buf * Cfg::kAccCols;
      for (int kb = 0; kb < args.num_k; ++kb, ++it) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (!mbar_wait(&conv_full[s], ph, abort_flag, args.st, 0x2201) ||
            !mbar_wait(&load_full[s], ph, abort_flag, args.st, 0x2202)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        const uint32_t xs = smem_u32(smem + s * Cfg::kStageBytes + Cfg::kOffX);
        const uint32_t ws = smem_u32(smem + s * Cfg::kStageBytes + Cfg::kOffW16);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint64_t xd = sdesc_sw128(xs + k * 32, 16, 1024);
#pragma unroll
          for (int p = 0; p < Cfg::kNumW16; ++p) {
            const uint64_t wd = sdesc_sw128(ws + p * Cfg::kW16Bytes + k * 2048, 8192, 1024);
            const uint32_t acc = (kb | k | p) != 0 ? 1u : 0u;
            if (kSwap) {
              umma_f16_ss(d_tmem, wd, xd, idesc, acc);
            } else {
              umma_f16_ss(d_tmem, xd, wd, idesc, acc);
            }
          }
        }
        umma_commit(&stage_empty[s]);
      }
      if (!aborted) umma_commit(&acc_full[buf]);
    }
    umma_commit(mma_done);
    DevStatus quiet = args.st;
    quiet.word = nullptr;
    mbar_wait(mma_done, 0, never_flag, quiet, 0);
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------- convert --
    const int ct = threadIdx.x - 128;  // 0..127
    int it = 0;
    bool ok_run = true;
    for (int t = blockIdx.x; t < num_tiles && ok_run; t += gridDim.x) {
      for (int kb = 0; kb < args.num_k; ++kb, ++it) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (!mbar_wait(&load_full[s], ph, abort_flag, args.st, 0x2300)) { ok_run = false; break; }
        uint8_t* st = smem + s * Cfg::kStageBytes;
        const uint8_t* raw = st + Cfg::kOffRaw;
        uint8_t* w16 = st + Cfg::kOffW16;
        if (kQ == kInt8) {
          // thread -> (k row r, n half h); raw unit u of row r sits at unit u ^ (r & 7)
          const int r = ct >> 1;
          const int h = ct & 1;
          const int sw = r & 7;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int u = 4 * h + i;
            const uint4 rv = *reinterpret_cast<const uint4*>(raw + r * 128 + ((u ^ sw) << 4));
            uint4 o0, o1;
            dequant_i8x16(rv, o0, o1);
            uint8_t* dst = w16 + h * 8192 + r * 128;
            *reinterpret_cast<uint4*>(dst + (((2 * i) ^ sw) << 4)) = o0;
            *reinterpret_cast<uint4*>(dst + (((2 * i + 1) ^ sw) << 4)) = o1;
          }
        } else {
          // thread -> (byte row kk: k rows 2kk and 2kk+1, n quarter qn: 32 channels)
          const int kk = ct >> 2;
          const int qn = ct & 3;
          const int swr = kk & 7;                 // swizzle of the raw row
          const int r0 = 2 * kk, r1 = 2 * kk + 1;  // fp16 rows
          const __half* sc = reinterpret_cast<const __half*>(st + Cfg::kOffScale) + qn * 32;
          const __half2 b8 = __float2half2_rn(1032.f);  // 1024 + 8
          uint8_t* hi = w16;
          uint8_t* lo = w16 + Cfg::kW16Bytes;
          const int chunk = qn >> 1;
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int u = 2 * qn + i;
            const uint4 rv = *reinterpret_cast<const uint4*>(raw + kk * 128 + ((u ^ swr) << 4));
            const uint32_t words[4] = {rv.x, rv.y, rv.z, rv.w};
            uint32_t hv0[8], lv0[8], hv1[8], lv1[8];  // rows r0 / r1, 16 channels each
#pragma unroll
            for (int wdx = 0; wdx < 4; ++wdx) {
              const uint32_t lo_n = (words[wdx] & 0x0F0F0F0Fu) ^ 0x08080808u;        // k even
              const uint32_t hi_n = ((words[wdx] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u; // k odd
              const __half2 s01 = *reinterpret_cast<const __half2*>(sc + i * 16 + wdx * 4);
              const __half2 s23 = *reinterpret_cast<const __half2*>(sc + i * 16 + wdx * 4 + 2);
#pragma unroll
              for (int half_sel = 0; half_sel < 2; ++half_sel) {
                const uint32_t sel = half_sel ? 0x7362u : 0x5140u;
                const __half2 s2 = half_sel ? s23 : s01;
                const __half2 q0 = __hsub2(u32_as_h2(bytes_to_h2(lo_n, sel)), b8);
                const __half2 q1 = __hsub2(u32_as_h2(bytes_to_h2(hi_n, sel)), b8);
                const __half2 w0h = __hmul2(q0, s2);
                const __half2 w1h = __hmul2(q1, s2);
                const __half2 w0l = __hfma2(q0, s2, __hneg2(w0h));
                const __half2 w1l = __hfma2(q1, s2, __hneg2(w1h));
                hv0[wdx * 2 + half_sel] = h2_as_u32(w0h);
                lv0[wdx * 2 + half_sel] = h2_as_u32(w0l);
                hv1[wdx * 2 + half_sel] = h2_as_u32(w1h);
                lv1[wdx * 2 + half_sel] = h2_as_u32(w1l);
              }
            }
            // 16 channels = two fp16 units; column within the chunk = 32 (qn & 1) + 16 i
            const int v0 = 4 * (qn & 1) + 2 * i;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int v = v0 + e;
              const int o0 = chunk * 8192 + r0 * 128 + ((v ^ (r0 & 7)) << 4);
              const int o1 = chunk * 8192 + r1 * 128 + ((v ^ (r1 & 7)) << 4);
              *reinterpret_cast<uint4*>(hi + o0) = make_uint4(hv0[4 * e], hv0[4 * e + 1], hv0[4 * e + 2], hv0[4 * e + 3]);
              *reinterpret_cast<uint4*>(lo + o0) = make_uint4(lv0[4 * e], lv0[4 * e + 1], lv0[4 * e + 2], lv0[4 * e + 3]);
              *reinterpret_cast<uint4*>(hi + o1) = make_uint4(hv1[4 * e], hv1[4 * e + 1], hv1[4 * e + 2], hv1[4 * e + 3]);
              *reinterpret_cast<uint4*>(lo + o1) = make_uint4(lv1[4 * e], lv1[4 * e + 1], lv1[4 * e + 2], lv1[4 * e + 3]);
            }
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv_full[s]);
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue --
    const uint32_t q = warp & 3;
    const int lrow = q * 32 + lane;  // TMEM lane: m (normal) or n (swap)
    const uint32_t lane_base = tmem + ((q * 32) << 16);
    int tc = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tc) {
      const int mb = t % args.num_m;
      const int nb = t / args.num_m;
      const int buf = tc & 1;
      const uint32_t use = tc >> 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], use & 1, abort_flag, args.st, 0x2400))) break;
      tc_fence_after();
      const uint32_t acc = lane_base + buf * Cfg::kAccCols;
      if (kSwap) {
        const int n = nb * kTileN + lrow;
        const float sc = (args.chan_scale != nullptr && n < args.N) ? __half2float(args.chan_scale[n]) : 1.f;
#pragma unroll
        for (int c = 0; c < (kNX + 31) / 32; ++c) {
          uint32_t r[32];
          if (kNX >= 32) {
            tmem_ld32(acc + c * 32, r);
          } else {
            uint32_t r16[16];
            tmem_ld16(acc, r16);
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = r16[i];
          }
          tmem_wait_ld();
          if (n < args.N) {
#pragma unroll
            for (int i = 0; i < (kNX >= 32 ? 32 : kNX); ++i) {
              const int m = c * 32 + i;
              if (m < args.M) args.Y[static_cast<int64_t>(m) * args.ldy + n] = __uint_as_float(r[i]) * sc;
            }
          }
        }
      } else {
        const int m = mb * 128 + lrow;
        float* yrow = args.Y + static_cast<int64_t>(m) * args.ldy;
#pragma unroll 1
        for (int c = 0; c < kTileN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(acc + c * 32, r);
          tmem_wait_ld();
          const int n0 = nb * kTileN + c * 32;
          if (m < args.M) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int n = n0 + i;
              if (n < args.N) {
                const float sc = args.chan_scale != nullptr ? __half2float(__ldg(args.chan_scale + n)) : 1.f;
                yrow[n] = __uint_as_float(r[i]) * sc;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

struct QProblem {
  const void* X;
  int64_t ldx;  // elements
  const void* W;
  int64_t ldw;  // bytes per stored row (int8: per k; int4: per pair of k)
  const void* scale;  // int8: [N] (nullable); int4: [K/128, N]
  int64_t lds;        // int4 scale row stride (elements)
  float* Y;
  int64_t ldy;
  int M, N, K;
  int kind;
};

template <int kQ, bool kSwap, int kNX>
int launch_wq(const QProblem& p, cudaStream_t stream) {
  using Cfg = QCfg<kQ, kSwap, kNX>;
  CUtensorMap tmX, tmW, tmS;
  {
    uint64_t dims[2] = {static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.M)};
    uint64_t strides[1] = {static_cast<uint64_t>(p.ldx) * 2};
    uint32_t box[2] = {64, static_cast<uint32_t>(kNX)};
    int rc = encode_tmap(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.X, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NESO_OK) return rc;
  }
  {
    const uint64_t rows = kQ == kInt8 ? p.K : p.K / 2;
    uint64_t dims[2] = {static_cast<uint64_t>(p.N), rows};
    uint64_t strides[1] = {static_cast<uint64_t>(p.ldw)};
    uint32_t box[2] = {128, kQ == kInt8 ? 64u : 32u};
    int rc = encode_tmap(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p.W, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NESO_OK) return rc;
  }
  if (kQ == kInt4G128) {
    uint64_t dims[2] = {static_cast<uint64_t>(p.N), static_cast<uint64_t>(p.K / 128)};
    uint64_t strides[1] = {static_cast<uint64_t>(p.lds) * 2};
    uint32_t box[2] = {128, 1};
    int rc = encode_tmap(&tmS, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.scale, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != NESO_OK) return rc;
  } else {
    tmS = tmX;  // unused
  }
  QArgs args{};
  args.Y = p.Y;
  args.ldy = p.ldy;
  args.chan_scale = kQ == kInt8 ? static_cast<const __half*>(p.scale) : nullptr;
  args.M = p.M;
  args.N = p.N;
  args.K = p.K;
  args.num_m = kSwap ? 1 : (p.M + 127) / 128;
  args.num_n = (p.N + kTileN - 1) / kTileN;
  args.num_k = (p.K + kBK - 1) / kBK;
  int rc = device_status(&args.st);
  if (rc != NESO_OK) return rc;
  const int tiles = args.num_m * args.num_n;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  auto kern = wq_gemm_kernel<kQ, kSwap, kNX>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(wq_gemm)");
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(tmX, tmW, tmS, args);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "wq_gemm launch");
  return ok();
}

template <int kQ>
int dispatch_wq(const QProblem& p, cudaStream_t stream) {
  if (p.M <= 16) return launch_wq<kQ, true, 16>(p, stream);
  if (p.M <= 32) return launch_wq<kQ, true, 32>(p, stream);
  if (p.M <= 64) return launch_wq<kQ, true, 64>(p, stream);
  return launch_wq<kQ, false, 128>(p, stream);
}

__global__ void zero_y_kernel(float* Y, int64_t ldy, int M, int N) {
  const int64_t total = static_cast<int64_t>(M) * N;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    Y[(i / N) * ldy + (i % N)] = 0.f;
  }
}

int run_wq(const QProblem& p, cudaStream_t stream) {
  if (p.M < 0 || p.N < 0 || p.K < 0) return fail(NESO_ERR_INVALID_ARG, "negative size");
  if (p.M == 0 || p.N == 0) return ok();
  if (p.Y == nullptr) return fail(NESO_ERR_INVALID_ARG, "null output");
  if (p.ldy < p.N) return fail(NESO_ERR_INVALID_ARG, "output row stride < N");
  if (p.K == 0) {
    zero_y_kernel<<<256, 256, 0, stream>>>(p.Y, p.ldy, p.M, p.N);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : cuda_fail(e, "zero launch");
  }
  if (p.X == nullptr || p.W == nullptr) return fail(NESO_ERR_INVALID_ARG, "null input");
  if (p.ldx < p.K) return fail(NESO_ERR_INVALID_ARG, "activation row stride < K");
  if ((p.ldx * 2) % 16 != 0) return fail(NESO_ERR_MISALIGNED, "activation row stride must be a multiple of 8");
  if (p.ldw % 16 != 0) return fail(NESO_ERR_MISALIGNED, "weight row stride must be a multiple of 16 bytes");
  if (p.kind == kInt8) {
    if (p.ldw < p.N) return fail(NESO_ERR_INVALID_ARG, "weight row stride < N");
    return dispatch_wq<kInt8>(p, stream);
  }
  if (p.K % 128 != 0) return fail(NESO_ERR_UNSUPPORTED, "int4 group-128 needs K %% 128 == 0 (K=%d)", p.K);
  if (p.scale == nullptr) return fail(NESO_ERR_INVALID_ARG, "null scales");
  if (p.lds < p.N || (p.lds * 2) % 16 != 0) return fail(NESO_ERR_MISALIGNED, "scale row stride must be >= N, multiple of 8");
  return dispatch_wq<kInt4G128>(p, stream);
}

}  // namespace
}  // namespace neso

using namespace neso;

extern "C" {

int neso_w8a16_matmul(const void* A, const int8_t* B, float* C, int32_t K, int32_t stride_am, int32_t stride_bk,
                      int32_t stride_cm, int32_t BM, int32_t BN, int32_t BK, uint32_t grid_x, uint32_t grid_y,
                      uint32_t grid_z, neso_stream_t stream) {
  return neso_w8a16_scaled_matmul(A, B, C, nullptr, K, stride_am, stride_bk, stride_cm, BM, BN, BK, grid_x, grid_y,
                                  grid_z, stream);
}

int neso_w8a16_scaled_matmul(const void* A, const int8_t* B, float* C, const void* scale, int32_t K,
                             int32_t stride_am, int32_t stride_bk, int32_t stride_cm, int32_t BM, int32_t BN,
                             int32_t BK, uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream) {
  if (BM <= 0 || BN <= 0 || BK <= 0) return fail(NESO_ERR_INVALID_ARG, "BM/BN/BK must be positive");
  if (grid_z != 1) return fail(NESO_ERR_GRID, "grid_z must be 1");
  // The reference has no M/N arguments and no masks: M = grid_x * BM, N = grid_y * BN.
  const int64_t M = static_cast<int64_t>(grid_x) * BM;
  const int64_t N = static_cast<int64_t>(grid_y) * BN;
  if (M > INT32_MAX || N > INT32_MAX) return fail(NESO_ERR_GRID, "grid implies an out-of-range M or N");
  if (stride_bk < N || stride_cm < N) return fail(NESO_ERR_GRID, "grid implies N=%lld wider than the row strides",
                                                  (long long)N);
  QProblem p{};
  p.X = A; p.ldx = stride_am;
  p.W = B; p.ldw = stride_bk;
  p.scale = scale; p.lds = 0;
  p.Y = C; p.ldy = stride_cm;
  p.M = static_cast<int>(M); p.N = static_cast<int>(N); p.K = K;
  p.kind = kInt8;
  return run_wq(p, as_stream(stream));
}

int neso_w8a16_matmul_mnk(const void* X, const int8_t* W, const void* scale, float* Y, int32_t M, int32_t N,
                          int32_t K, neso_stream_t stream) {
  QProblem p{};
  p.X = X; p.ldx = K;
  p.W = W; p.ldw = N;
  p.scale = scale; p.lds = 0;
  p.Y = Y; p.ldy = N;
  p.M = M; p.N = N; p.K = K;
  p.kind = kInt8;
  return run_wq(p, as_stream(stream));
}

int neso_w4a16_g128_matmul(const void* X, const uint8_t* Wq, const void* scales, float* Y, int32_t M, int32_t N,
                           int32_t K, neso_stream_t stream) {
  QProblem p{};
  p.X = X; p.ldx = K;
  p.W = Wq; p.ldw = N;
  p.scale = scales; p.lds = N;
  p.Y = Y; p.ldy = N;
  p.M = M; p.N = N; p.K = K;
  p.kind = kInt4G128;
  return run_wq(p, as_stream(stream));
}

}  // extern "C"
