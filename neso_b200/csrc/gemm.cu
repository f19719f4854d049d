// Dense fp16 GEMM C[M,N] (fp32) = A[M,K] (fp16) . B[K,N] (fp16), fp32 accumulation.
//
// Reference kernels: tests/test_aot.py:70-99 (matmul_kernel with M/N/K and
// strides), bench/bench_matmul.py:77-153 (TTIR matmul_kernel(a,b,c,K,...)),
// bench/bench_matmul_opt.py:129-139 (hand MSL matmul_opt, half in / float out).
//
// B200 design (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A tile [128 x 64] K-major, B tile [64 x BN]
//               MN-major (B is row-major [K,N]), both 128-byte swizzled, into
//               a STAGES-deep shared-memory ring guarded by full/empty mbarriers.
//   warp 1      single-thread tcgen05.mma issuer, M=128 x N=BN x K=16 per
//               instruction, fp32 accumulator in TMEM, double-buffered so the
//               epilogue of tile i overlaps the mainloop of tile i+1.
//   warp 2      TMEM allocator.
//   warps 4-7   epilogue: tcgen05.ld 32 lanes x 32 columns -> registers ->
//               fp32 C rows in global memory.
// Large problems use 256 x 256 tiles instead: each stage holds two 128-row A
// tiles and one B tile, warp 1 issues two M=128 N=256 MMAs per K step (one per
// accumulator, 512 TMEM columns, single-buffered) and warps 4-11 drain the two
// accumulators between tiles. Every B byte then feeds 256 rows, cutting the
// L2 -> SM operand traffic per FLOP by a third.
// Ragged M/N/K edges come from TMA zero fill on loads and masked stores.
#include "runtime.h"

namespace neso {
namespace {

constexpr int kBM = 128;  // rows per accumulator (one M = 128 MMA)
constexpr int kBK = 64;
constexpr int kGroupM = 16;  // L2 rasterisation: 16 M-tiles share a B column panel

// MH = 128-row accumulators per tile. MH = 2: a 256 x BN tile whose B stage
// feeds two M = 128 MMAs, so each operand byte brought from L2 serves twice the
// FLOPs of a 128-row tile; the two accumulators fill TMEM, so there is one
// accumulator buffer and the epilogue (8 warps) runs between tiles.
template <int BN, int MH = 1>
struct GemmCfg {
  static constexpr int kThreads = 128 + 128 * MH;
  static constexpr int kTileM = kBM * MH;
  static constexpr int kStages = MH == 2 ? 3 : (BN >= 256) ? 4 : 6;
  static constexpr int kABytes = kTileM * kBK * 2;  // 16 KB per 128 rows
  static constexpr int kBBytes = kBK * BN * 2;      // 8 KB per 64 columns
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kAccBufs = MH == 2 ? 1 : 2;
  static constexpr int kTmemCols = kAccBufs * MH * BN;
  // C staging: 32 rows x 32 fp32 per epilogue warp, double-buffered for
  // 128-row tiles (a store of one block overlaps loading the next), single
  // for 256 x 256 tiles, whose stages fill the rest of shared memory.
  static constexpr int kOutBufs = MH == 1 ? 2 : 1;
  static constexpr int kOutBytes = 4 * MH * 4096 * kOutBufs;
  static constexpr int kSmemBytes = kStages * kStageBytes + kOutBytes + 1024 /*align*/ + 256 /*barriers*/;
};

struct GemmArgs {
  float* C;
  int64_t ldc;
  int M, N, K;
  int num_m, num_n, num_k;
  int b_chunked;  // B tile loaded with one 3-D TMA (all BN/64 column chunks)
  int c_tma;      // C written by TMA stores (16-byte aligned base and row stride)
  DevStatus st;
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = kGroupM * num_n;
  const int g = t / per_group;
  const int first_m = g * kGroupM;
  const int gsize = min(num_m - first_m, kGroupM);
  const int r = t - g * per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

template <int BN, int MH>
__global__ void __launch_bounds__(GemmCfg<BN, MH>::kThreads, 1)
    gemm_f16_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmB3, const __grid_constant__ CUtensorMap tmC,
                            GemmArgs args) {
  using Cfg = GemmCfg<BN, MH>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                       // S x MH x 16 KB
  uint8_t* sB = smem + S * Cfg::kABytes;    // S x (BN/64) x 8 KB
  uint8_t* sOut = smem + S * Cfg::kStageBytes;  // 4 KB per epilogue warp and staging buffer
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + Cfg::kOutBytes);
  uint64_t* full = bars;                    // [S]
  uint64_t* empty = bars + S;               // [S]
  uint64_t* acc_full = bars + 2 * S;        // [2]
  uint64_t* acc_empty = bars + 2 * S + 2;   // [2]
  uint64_t* mma_done = bars + 2 * S + 4;    // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* never_flag = abort_flag + 1;  // stays 0: drain waits ignore the abort

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int num_tiles = args.num_m * args.num_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4 * MH);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    *never_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmB3);
    if (args.c_tma) tma_prefetch_desc(&tmC);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: nothing global is read or written before
  // the previous kernel on the stream has completed.
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------- producer --
    int it = 0;
    bool aborted = false;
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, args.num_m, args.num_n, mb, nb);
      for (int kb = 0; kb < args.num_k; ++kb, ++it) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, args.st, 0x100)) {
          aborted = true;
          break;
        }
        mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
#pragma unroll
        for (int h = 0; h < MH; ++h) {
          tma_load_2d(sA + s * Cfg::kABytes + h * (kBM * kBK * 2), &tmA, &full[s], kb * kBK, mb * Cfg::kTileM + h * kBM);
        }
        if (args.b_chunked) {
          tma_load_3d(sB + s * Cfg::kBBytes, &tmB3, &full[s], 0, kb * kBK, nb * (BN / 64));
        } else {
#pragma unroll
          for (int c = 0; c < BN / 64; ++c) {
            tma_load_2d(sB + s * Cfg::kBBytes + c * 8192, &tmB, &full[s], nb * BN + c * 64, kb * kBK);
          }
        }
      }
    }
    if (aborted) {
      // Drain this CTA's own copies still in flight before the CTA exits.
      DevStatus quiet = args.st;
      quiet.word = nullptr;
      for (int i = (it > S ? it - S : 0); i < it; ++i) {
        mbar_wait(&full[i % S], (i / S) & 1, never_flag, quiet, 0);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------- MMA issuer --
    constexpr uint32_t idesc = idesc_f16_f32(kBM, BN, 0, 1);
    int it = 0, tc = 0;
    bool aborted = false;
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x, ++tc) {
      const int buf = tc % Cfg::kAccBufs;
      const uint32_t use = tc / Cfg::kAccBufs;
      if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, abort_flag, args.st, 0x200)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * MH * BN;
      for (int kb = 0; kb < args.num_k; ++kb, ++it) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag, args.st, 0x201)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * Cfg::kABytes);
        const uint32_t b0 = smem_u32(sB + s * Cfg::kBBytes);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint64_t bd = sdesc_sw128(b0 + k * 2048, 8192, 1024);
#pragma unroll
          for (int h = 0; h < MH; ++h) {
            const uint64_t ad = sdesc_sw128(a0 + h * (kBM * kBK * 2) + k * 32, 16, 1024);
            umma_f16_ss(d_tmem + h * BN, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
        }
        umma_commit(&empty[s]);
      }
      if (!aborted) umma_commit(&acc_full[buf]);
    }
    // Every MMA this thread issued must be complete before TMEM is freed.
    umma_commit(mma_done);
    DevStatus quiet = args.st;
    quiet.word = nullptr;
    mbar_wait(mma_done, 0, never_flag, quiet, 0);
  } else if (warp >= 4) {
    // --------------------------------------------------------- epilogue --
    const uint32_t q = warp & 3;  // TMEM lane quarter this warp may access
    const int h = (warp - 4) >> 2;  // accumulator (128-row half of the tile)
    const int row_in_tile = h * kBM + q * 32 + lane;
    const bool vec_ok = (args.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(args.C) & 15u) == 0);
    int tc = 0;
    int nstore = 0;  // TMA stores issued by this warp
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tc) {
      int mb, nb;
      tile_coords(t, args.num_m, args.num_n, mb, nb);
      const int buf = tc % Cfg::kAccBufs;
      const uint32_t use = tc / Cfg::kAccBufs;
      // Warp-uniform: every lane must agree before the .sync.aligned TMEM loads.
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], use & 1, abort_flag, args.st, 0x300))) break;
      tc_fence_after();
      if (args.c_tma) {
        // TMEM -> registers -> this warp's 128-byte-swizzled staging rows ->
        // one TMA store per 32 x 32 block: full-line writes, and the
        // accumulator is released as soon as its last columns are loaded.
        const int row0 = mb * Cfg::kTileM + h * kBM + q * 32;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem_base + ((q * 32) << 16) + (buf * MH + h) * BN + c * 32, r);
          tmem_wait_ld();
          if (c == BN / 32 - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
          }
          const int col0 = nb * BN + c * 32;
          if (row0 >= args.M || col0 >= args.N) continue;  // warp-uniform: block wholly past C
          // Staging blocks alternate by stores issued, so the block written
          // here is the one the store before last read: with two blocks, the
          // last store may still be reading the other. (Alternating by block
          // index instead let a block skipped past the edge of C hand the
          // next write the block the last store was still reading.)
          uint8_t* stage = sOut + ((warp - 4) * Cfg::kOutBufs + (nstore++ % Cfg::kOutBufs)) * 4096;
          if (lane == 0) {
            if (Cfg::kOutBufs == 2) {
              bulk_wait_read_but1();
            } else {
              bulk_wait_read_all();
            }
          }
          __syncwarp();
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            *reinterpret_cast<uint4*>(stage + lane * 128 + ((v ^ (lane & 7)) << 4)) =
                make_uint4(r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, stage, col0, row0);
            bulk_commit();
          }
        }
        continue;
      }
      const int grow = mb * Cfg::kTileM + row_in_tile;
      float* crow = args.C + static_cast<int64_t>(grow) * args.ldc;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((q * 32) << 16) + (buf * MH + h) * BN + c * 32, r);
        tmem_wait_ld();
        const int col0 = nb * BN + c * 32;
        if (grow < args.M) {
          if (vec_ok && col0 + 32 <= args.N) {
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              float4 f = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                     __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
              *reinterpret_cast<float4*>(crow + col0 + 4 * v) = f;
            }
          } else {
#pragma unroll
            for (int v = 0; v < 32; ++v) {
              if (col0 + v < args.N) crow[col0 + v] = __uint_as_float(r[v]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (lane == 0) bulk_wait_all();  // this warp's C stores are complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// Zero C when K == 0 (the accumulator is never written).
__global__ void zero_rows_kernel(float* C, int64_t ldc, int M, int N) {
  const int64_t total = static_cast<int64_t>(M) * N;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    C[(i / N) * ldc + (i % N)] = 0.f;
  }
}

template <int BN, int MH = 1>
int launch_gemm_bn(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc, int M, int N, int K,
                   cudaStream_t stream) {
  using Cfg = GemmCfg<BN, MH>;
  CUtensorMap tmA, tmB;
  {
    uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
    uint32_t box[2] = {64, 128};
    int rc = encode_tmap(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NESO_OK) return rc;
  }
  {
    uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K)};
    uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
    uint32_t box[2] = {64, 64};
    int rc = encode_tmap(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, B, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NESO_OK) return rc;
  }
  // B as [N/64 chunks][K rows][64 columns]: one TMA per stage fetches all
  // BN/64 chunks of a tile. Only when N is a whole number of chunks, so the
  // last chunk never reaches past the end of a row.
  CUtensorMap tmB3 = tmB;
  int b_chunked = 0;
  if (N % 64 == 0) {
    uint64_t dims[3] = {64, static_cast<uint64_t>(K), static_cast<uint64_t>(N / 64)};
    uint64_t strides[2] = {static_cast<uint64_t>(ldb) * 2, 128};
    uint32_t box[3] = {64, 64, BN / 64};
    int rc = encode_tmap(&tmB3, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, B, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NESO_OK) return rc;
    b_chunked = 1;
  }
  // C through TMA stores when its base and row stride are 16-byte aligned.
  CUtensorMap tmC = tmA;
  int c_tma = 0;
  if (ldc % 4 == 0 && (reinterpret_cast<uintptr_t>(C) & 15u) == 0) {
    uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
    uint64_t strides[1] = {static_cast<uint64_t>(ldc) * 4};
    uint32_t box[2] = {32, 32};
    int rc = encode_tmap(&tmC, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, C, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NESO_OK) return rc;
    c_tma = 1;
  }
  GemmArgs args{};
  args.b_chunked = b_chunked;
  args.c_tma = c_tma;
  args.C = C;
  args.ldc = ldc;
  args.M = M;
  args.N = N;
  args.K = K;
  args.num_m = (M + Cfg::kTileM - 1) / Cfg::kTileM;
  args.num_n = (N + BN - 1) / BN;
  args.num_k = (K + kBK - 1) / kBK;
  int rc = device_status(&args.st);
  if (rc != NESO_OK) return rc;
  const int tiles = args.num_m * args.num_n;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  auto kern = gemm_f16_tcgen05_kernel<BN, MH>;
  {
    int src = kernel_setup(reinterpret_cast<const void*>(kern), Cfg::kSmemBytes, nullptr);
    if (src != NESO_OK) return src;
  }
  cudaError_t e = launch_pdl(kern, dim3(grid), dim3(Cfg::kThreads), Cfg::kSmemBytes, stream, tmA, tmB, tmB3, tmC, args);
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  return ok();
}

// Output tile shape: score = wave efficiency (tiles / (waves * SMs)) weighted
// by the per-tile efficiency of larger tiles (less operand traffic per FLOP).
// Returns the tile width, or 512 for the 256 x 256 tile (two accumulators).
int pick_tile_n(int M, int N, int sms) {
  const int cands[4] = {512, 256, 128, 64};
  // Relative throughput of each tile at full occupancy, measured on B200
  // (square fp16 GEMMs, 2048-8192): N=256 MMAs hide operand traffic best, and
  // 256 x 256 tiles (each B stage feeding two MMAs) are 7 % faster again
  // (4096: 1143 -> 1218, 8192: 1276 -> 1374 TFLOP/s at equal wave counts).
  const double weight[4] = {1.07, 1.0, 0.72, 0.5};
  int best = 64;
  double best_score = -1.0;
  for (int i = 0; i < 4; ++i) {
    const int bn = cands[i] == 512 ? 256 : cands[i];
    const int tm = cands[i] == 512 ? 2 * kBM : kBM;
    if (bn > 64 && N <= bn / 2) continue;  // mostly empty tile
    if (tm > kBM && M <= kBM) continue;
    const int64_t num_m = (M + tm - 1) / tm;
    const int64_t tiles = num_m * ((N + bn - 1) / bn);
    const int64_t waves = (tiles + sms - 1) / sms;
    const double score = weight[i] * static_cast<double>(tiles) / static_cast<double>(waves * sms);
    if (score > best_score + 1e-9) {
      best_score = score;
      best = cands[i];
    }
  }
  return best;
}

}  // namespace

// Shared entry used by every GEMM-shaped C-ABI function.
int gemm_f16_f32(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc, int M, int N, int K,
                 cudaStream_t stream) {
  if (M < 0 || N < 0 || K < 0) return fail(NESO_ERR_INVALID_ARG, "negative size M=%d N=%d K=%d", M, N, K);
  if (M == 0 || N == 0) return ok();
  if (C == nullptr || (K > 0 && (A == nullptr || B == nullptr))) return fail(NESO_ERR_INVALID_ARG, "null pointer");
  if (ldc < N) return fail(NESO_ERR_INVALID_ARG, "stride_cm %lld < N %d", (long long)ldc, N);
  if (K == 0) {
    zero_rows_kernel<<<256, 256, 0, stream>>>(C, ldc, M, N);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : cuda_fail(e, "zero launch");
  }
  if (lda < K || ldb < N) return fail(NESO_ERR_INVALID_ARG, "row stride smaller than the row");
  if ((lda * 2) % 16 != 0 || (ldb * 2) % 16 != 0) {
    return fail(NESO_ERR_MISALIGNED, "fp16 row strides must be multiples of 8 elements (lda=%lld ldb=%lld)",
                (long long)lda, (long long)ldb);
  }
  const int bn = pick_tile_n(M, N, sm_count());
  if (bn == 512) return launch_gemm_bn<256, 2>(A, lda, B, ldb, C, ldc, M, N, K, stream);
  if (bn == 256) return launch_gemm_bn<256>(A, lda, B, ldb, C, ldc, M, N, K, stream);
  if (bn == 128) return launch_gemm_bn<128>(A, lda, B, ldb, C, ldc, M, N, K, stream);
  return launch_gemm_bn<64>(A, lda, B, ldb, C, ldc, M, N, K, stream);
}

}  // namespace neso

using namespace neso;

extern "C" {

int neso_matmul_kernel(const void* a, const void* b, float* c, int32_t M, int32_t N, int32_t K, int32_t stride_am,
                       int32_t stride_ak, int32_t stride_bk, int32_t stride_bn, int32_t stride_cm, int32_t stride_cn,
                       int32_t BLOCK_M, int32_t BLOCK_N, int32_t BLOCK_K, uint32_t grid_x, uint32_t grid_y,
                       uint32_t grid_z, neso_stream_t stream) {
  if (BLOCK_M <= 0 || BLOCK_N <= 0 || BLOCK_K <= 0) return fail(NESO_ERR_INVALID_ARG, "BLOCK_* must be positive");
  if (M < 0 || N < 0 || K < 0) return fail(NESO_ERR_INVALID_ARG, "negative size");
  const uint32_t gm = static_cast<uint32_t>((M + BLOCK_M - 1) / BLOCK_M);
  const uint32_t gn = static_cast<uint32_t>((N + BLOCK_N - 1) / BLOCK_N);
  if (grid_x != gm || grid_y != gn || grid_z != 1) {
    return fail(NESO_ERR_GRID, "grid (%u,%u,%u) != (cdiv(M,BLOCK_M)=%u, cdiv(N,BLOCK_N)=%u, 1)", grid_x, grid_y,
                grid_z, gm, gn);
  }
  if (stride_ak != 1 || stride_bn != 1 || stride_cn != 1) {
    return fail(NESO_ERR_UNSUPPORTED, "only unit inner strides are supported (stride_ak=%d stride_bn=%d "
                                      "stride_cn=%d)", stride_ak, stride_bn, stride_cn);
  }
  return gemm_f16_f32(a, stride_am, b, stride_bk, c, stride_cm, M, N, K, as_stream(stream));
}

int neso_matmul_tiled(const void* a, const void* b, float* c, int32_t K, int32_t stride_am, int32_t stride_bk,
                      int32_t stride_cm, int32_t BM, int32_t BN, uint32_t grid_x, uint32_t grid_y, uint32_t grid_z,
                      neso_stream_t stream) {
  if (BM <= 0 || BN <= 0) return fail(NESO_ERR_INVALID_ARG, "BM/BN must be positive");
  if (grid_z != 1) return fail(NESO_ERR_GRID, "grid_z must be 1");
  const int64_t M = static_cast<int64_t>(grid_x) * BM;
  const int64_t N = static_cast<int64_t>(grid_y) * BN;
  if (M > INT32_MAX || N > INT32_MAX) return fail(NESO_ERR_GRID, "grid implies an out-of-range M or N");
  return gemm_f16_f32(a, stride_am, b, stride_bk, c, stride_cm, static_cast<int>(M), static_cast<int>(N), K,
                      as_stream(stream));
}

}  // extern "C"
