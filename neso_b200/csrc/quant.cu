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
//   warp 0      TMA: raw weight tile(s) (int8 [64 k][128 n] or packed int4
//               [32 byte-rows][128 n], 128-byte swizzled) and (int4, M >= 129)
//               the group's fp16 scale row; warp 3: TMA of the activation tile
//               (and, int4 M >= 129, of its E5M2 copy, 64-byte swizzled).
//   warps 4-7,  dequantise raw -> fp16 directly into the MN-major 128-byte
//   12-15       swizzled layout tcgen05 reads; fence.proxy.async; arrive. The
//               two groups take alternate K blocks (or, with two channel
//               tiles per unit, one tile each of every K block).
//                 int8: exact, (b ^ 0x80) | 0x6400 as fp16 is 1024 + b + 128.
//                 int4, M >= 129 layout: q exact the same way, then w = q * s
//                 is split into w_hi = fp16(q * s) and w_lo = fma(q, s, -w_hi)
//                 (the exact rounding error, at most 3 significant bits),
//                 stored as E5M2 of 2^8 w_lo (exact), so the MMAs sum q * s
//                 up to the E5M2 rounding of X in the w_lo term.
//                 int4, swapped layout (M <= 128): q only (exact in fp16); the group
//                 scale is applied to fp32 partial sums instead (below).
//   warp 1      tcgen05.mma issuer (kind::f16, fp32 accumulators in TMEM);
//               int4 M >= 129 adds two kind::f8f6f4 MMAs (K = 32) per K
//               block for w_lo against an E5M2 copy of 2^-8 X (written by
//               a conversion kernel before the matmul); int4 M <= 128
//               accumulates each run of K blocks inside one 128-wide scale
//               group into its own buffer (double-buffered), so the epilogue
//               applies that group's scales while the next run accumulates.
//   warp 2      (int4, M <= 128) TMA producer of each run's scale row.
//   warps 8-11  epilogue: TMEM -> registers -> (int8: * f32(scale[n])) ->
//               swizzled staging -> TMA stores of Y (M >= 65 layout), or
//               direct coalesced stores (swapped layout). int4 swapped: the
//               running sums stay in registers, += partial * scale[g][n]
//               (M = 65..128: 128 sums a thread, the epilogue warpgroup
//               takes registers from warpgroup 0 with setmaxnreg).
// Orientation: M >= 65 computes Y units of 128 or 256 rows x 128 or 256
// channels (a host cost model picks the shape and any K split) with X as the
// A operand; M <= 64 (int4: M <= 128) swaps operands (A = dequantised W^T
// with M' = 128 output channels, B = X with N' = M rounded up to
// 16/32/64/128) so decode-sized batches still run on the tensor cores and the
// weight stream stays at HBM speed.
#include <algorithm>
#include <mutex>

#include "runtime.h"

namespace neso {
namespace {

constexpr int kThreads = 512;  // warps 12-15: second convert group
constexpr int kBK = 64;
constexpr int kTileN = 128;  // output channels per tile

enum QuantKind : int { kInt8 = 0, kInt4G128 = 1 };

template <int kQ, bool kSwap, int kNX, int kNT = 1>
struct QCfg {
  // kNT = 128-channel weight tiles per unit (2: both convert groups take one
  // tile of every K block and the X tile is used for 256 output channels,
  // halving the activation traffic per FLOP; large M only). kNX = activation
  // rows per unit: 128, or 256 in the M >= 65 layout (two 128-row
  // accumulators, each fp16 weight stage feeds two MMAs per K step, one
  // accumulator buffer).
  // Three decoupled rings so weight bytes stay in flight independently of
  // the dequant and MMA rate:
  //   R  raw weight tiles (int8 [64 k][128 n] or packed int4 [32][128] plus,
  //      int4 M >= 129, the group's 128 fp16 scales), deep: TMA -> convert warps;
  //   X  activation tiles [kNX rows][64 k] fp16: TMA -> MMA;
  //   F  dequantised fp16 weight tiles (int4 M >= 129: the fp16 w_hi tiles
  //      followed by the E5M2 w_lo tiles): convert -> MMA.
  // int4 swapped layout (kGS, group-scaled partial sums) adds a ring of scale rows
  // (one 128-channel row per tile and group run): TMA -> epilogue.
  static constexpr bool kGS = kQ == kInt4G128 && kSwap;
  // int4, M >= 65 layout (M >= 129): w = q * s is carried as w_hi = fp16(q * s) (kind::f16
  // MMAs) plus its exact remainder w_lo, which has at most 3 significant bits
  // and so is exact as E5M2 once scaled by 2^8; the w_lo MMAs run as
  // kind::f8f6f4 (twice the fp16 rate) against an E5M2 copy of X scaled by
  // 2^-8, appended to each X stage.
  static constexpr bool kF8Lo = kQ == kInt4G128 && !kSwap;
  // int4 swapped layout with 128 activation rows (M = 65..128): each
  // epilogue thread keeps 128 running sums, so warpgroup 2 (the epilogue)
  // grows to kRegsEpi registers and warpgroup 0 (TMA, MMA issuer) shrinks to
  // kRegsLow; the two convert warpgroups keep the launch's 128.
  static constexpr bool kWideEpi = kGS && kNX * kNT > 64;
  static constexpr uint32_t kRegsLow = 80;
  static constexpr uint32_t kRegsEpi = 176;
  static_assert(!kWideEpi || kRegsLow + kRegsEpi == 2 * 128, "register split must fit the launch pool");
  static constexpr int kRawTileBytes = (kQ == kInt8) ? 64 * 128 : kGS ? 32 * 128 : 32 * 128 + 1024;
  static constexpr int kRawBytes = kNT * kRawTileBytes;
  // 64-deep K blocks per fp16 weight (F) and activation (X) stage: two in the
  // swapped layout with paired tiles or int4, whose per-stage hand-offs
  // (barrier waits, the proxy fence, commits) otherwise cost as much as its
  // small MMAs (measured: W8A16 M=16 19.3 -> 17.8 us, W4A16 M=16/32/64
  // 21.1 / 25.5 / 30.6 -> 19.9 / 23.2 / 28.8 us; single-tile W8A16 M=32/64
  // measured slower, 20.9 / 22.9 -> 21.8 / 23.4); raw tiles stay one K block.
  static constexpr int kFKB = (kSwap && (kNT == 2 || kQ == kInt4G128)) ? 2 : 1;
  static constexpr int kXBlockBytes = kNX * kBK * 2;
  static constexpr int kX8Bytes = kF8Lo ? kNX * kBK : 0;  // E5M2 X block: kNX rows x 64 bytes, 64-byte swizzle
  static constexpr int kXBytes = kFKB * kXBlockBytes + kX8Bytes;
  static constexpr int kW16BlockBytes = kBK * kTileN * 2;      // 16 KB: one K block of one tile
  static constexpr int kW16Bytes = kFKB * kW16BlockBytes;      // one fp16 copy of one tile
  static constexpr int kLoBlockBytes = kBK * kTileN;  // 8 KB: one K block of one tile's E5M2 w_lo
  // Convert groups (warps 4-7, 12-15). A group's per-stage cost is mostly
  // fixed (barrier waits, the proxy fence, loop control: ~1300 cycles per
  // stage measured at M = 16), so the swapped layout lets each group take
  // alternate stages and convert every tile of its stage; the M >= 65 paired
  // layout keeps one tile per group on every stage.
  static constexpr bool kAltStages = kSwap || kNT == 1;
  static constexpr int kGroupTiles = kSwap ? kNT : 1;
  static constexpr int kConvGroupsPerStage = kAltStages ? 1 : kNT;
  static constexpr int kScSlots = kGS ? 16 : 0;
  static constexpr int kScBytes = kNT * 256;
  static constexpr int kFTileBytes = kW16Bytes + (kF8Lo ? kLoBlockBytes : 0);
  static constexpr int kFBytes = kNT * kFTileBytes;
  // kNX = 256 in the M >= 65 layout: 256-row units, two 128-row accumulators
  // (every fp16 weight stage feeds two MMAs per K step).
  static constexpr int kRowHalves = kSwap ? 1 : kNX / 128;
  static constexpr int kFStages = kSwap ? (kFKB == 1 ? 4 : kNT == 2 ? 2 : 3)
                                  : kRowHalves == 2 ? 2 : kNT == 2 ? (kQ == kInt8 ? 3 : 2) : (kQ == kInt4G128) ? 3 : 4;
  // X tiles come from L2 with about 2500 cycles of copy latency: a deep
  // ring keeps the MMAs fed when every K block needs a new 16 KB X tile.
  // Swapped layout: X tiles are 2-8 KB and the X ring moves in step with the
  // F ring (same depth, released by the same commit; deeper X rings measured
  // no faster at M = 16).
  static constexpr int kXStages = kSwap ? kFStages : kRowHalves == 2 ? 3 : kNT == 2 ? (kQ == kInt8 ? 4 : 3)
                                  : kF8Lo ? 4 : 6;
  static constexpr int kBudget = 224 * 1024;
  // Y staging for TMA stores (M >= 65 layout): 16 rows x 32 fp32 per epilogue
  // warp, two blocks (one store's read overlaps filling the next) where the
  // raw ring keeps its minimum depth.
  static constexpr int kMinRStages = kNT == 2 ? 3 : 4;
  static constexpr int kOutBufs =
      (kBudget - 4 * 2048 * 2 - kScSlots * kScBytes - kFStages * kFBytes - kXStages * kXBytes) / kRawBytes >= kMinRStages
          ? 2
          : 1;
  static constexpr int kOutBytes = kSwap ? 0 : 4 * 2048 * kOutBufs;
  static constexpr int kRStagesFit =
      (kBudget - kOutBytes - kScSlots * kScBytes - kFStages * kFBytes - kXStages * kXBytes) / kRawBytes;
  static constexpr int kRStages = kRStagesFit > 16 ? 16 : kRStagesFit;
  static constexpr int kOffR = 0;
  static constexpr int kOffX = kRStages * kRawBytes;
  static constexpr int kOffF = kOffX + kXStages * kXBytes;
  static constexpr int kOffOut = kOffF + kFStages * kFBytes;
  static constexpr int kOffSc = kOffOut + kOutBytes;
  static constexpr int kOffBars = kOffSc + kScSlots * kScBytes;
  static constexpr int kRawTx = kNT * ((kQ == kInt8) ? 64 * 128 : kGS ? 32 * 128 : 32 * 128 + 256);
  static constexpr int kAccCols = kSwap ? kNT * kNX : kRowHalves * kNT * kTileN;  // accumulator columns per buffer
  static constexpr int kAccBufs = 2 * kAccCols <= 512 ? 2 : 1;
  static_assert(!kGS || kAccBufs == 2, "group runs need two accumulator buffers");
  static constexpr int kTmemCols = (kAccBufs * kAccCols <= 32) ? 32 : (kAccBufs * kAccCols <= 64) ? 64
                                   : (kAccBufs * kAccCols <= 128) ? 128 : (kAccBufs * kAccCols <= 256) ? 256 : 512;
  static constexpr int kSmemBytes = kOffBars + 1024 + 1024;
  static_assert(kRStages >= kMinRStages, "raw ring too shallow");
  static_assert(kXBytes % 1024 == 0 && kRawBytes % 1024 == 0 && kFBytes % 1024 == 0, "1024-aligned stages");
};

struct QArgs {
  float* Y;
  int64_t ldy;
  const __half* chan_scale;  // int8: per-channel scale [N] (nullable)
  const float* tensor_scale;  // int8: one fp32 scale for the whole output (nullable; exclusive with chan_scale)
  float* partial;            // split-K: [splits][M][N] fp32 partial sums, else null
  int M, N, K;
  int num_m, num_n, num_k;
  int splits, kb_per_split;  // K blocks are split into `splits` ranges
  int y_tma;                 // Y / partial sums written by TMA stores (M >= 65 layout, aligned rows)
  DevStatus st;
};

// One work unit = (M tile, N tile, K range). K-split index fastest so the
// units of one output tile run side by side and share X in L2.
struct QUnit {
  int mb, nb, ks, kb0, kb1;
};
__device__ __forceinline__ QUnit unit_of(int t, const QArgs& a) {
  QUnit u;
  u.ks = t % a.splits;
  const int r = t / a.splits;
  u.mb = r % a.num_m;
  u.nb = r / a.num_m;
  u.kb0 = u.ks * a.kb_per_split;
  u.kb1 = min(a.num_k, u.kb0 + a.kb_per_split);
  return u;
}

// int4: the K blocks of a unit are accumulated in runs that stay inside one
// 128-wide scale group (two 64-deep K blocks); a unit's K range may start or
// end inside a group (K splits), which only shortens a run.
__device__ __forceinline__ bool run_starts(int kb, int kb0) { return kb == kb0 || (kb & 1) == 0; }
__device__ __forceinline__ bool run_ends(int kb, int kb1) { return kb + 1 == kb1 || (kb & 1) == 1; }

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

template <int kQ, bool kSwap, int kNX, int kNT>
__global__ void __launch_bounds__(kThreads, 1)
    wq_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmY,
                   const __grid_constant__ CUtensorMap tmX8, QArgs args) {
  using Cfg = QCfg<kQ, kSwap, kNX, kNT>;
  constexpr int kUnitN = kNT * kTileN;  // output channels per unit
  constexpr int RS = Cfg::kRStages, XS = Cfg::kXStages, FS = Cfg::kFStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sR = smem + Cfg::kOffR;
  uint8_t* sX = smem + Cfg::kOffX;
  uint8_t* sF = smem + Cfg::kOffF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBars);
  uint64_t* r_full = bars;              // [RS] raw tile landed (TMA)
  uint64_t* r_empty = r_full + RS;      // [RS] raw tile read by the 4 convert warps
  uint64_t* x_full = r_empty + RS;      // [XS] activation tile landed (TMA)
  uint64_t* x_empty = x_full + XS;      // [XS] MMAs done with it
  uint64_t* f_full = x_empty + XS;      // [FS] fp16 weights written (4 convert warps)
  uint64_t* f_empty = f_full + FS;      // [FS] MMAs done with them
  uint64_t* acc_full = f_empty + FS;    // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2] (the epilogue warps)
  uint64_t* mma_done = acc_empty + 2;
  uint64_t* sc_full = mma_done + 1;           // [kScSlots] int4 scale rows landed
  uint64_t* sc_empty = sc_full + Cfg::kScSlots;  // [kScSlots] epilogue done with them
  uint8_t* sSc = smem + Cfg::kOffSc;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sc_empty + Cfg::kScSlots);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* never_flag = abort_flag + 1;  // stays 0: drain waits ignore the abort

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int num_units = args.num_m * args.num_n * args.splits;

  if (threadIdx.x == 0) {
    for (int i = 0; i < RS; ++i) {
      mbar_init(&r_full[i], 1);
      mbar_init(&r_empty[i], 4 * Cfg::kConvGroupsPerStage);
    }
    for (int i = 0; i < XS; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < FS; ++i) {
      mbar_init(&f_full[i], 4 * Cfg::kConvGroupsPerStage);
      mbar_init(&f_empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(mma_done, 1);
    for (int i = 0; i < Cfg::kScSlots; ++i) {
      mbar_init(&sc_full[i], 1);
      mbar_init(&sc_empty[i], 4);
    }
    *abort_flag = 0;
    *never_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
    if (kQ == kInt4G128) tma_prefetch_desc(&tmS);
    if (Cfg::kF8Lo) tma_prefetch_desc(&tmX8);
    if (args.y_tma) tma_prefetch_desc(&tmY);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent launch: nothing global is read or written before
  // the previous kernel on the stream has completed.
  pdl_launch_dependents();
  pdl_wait();
  DevStatus quiet = args.st;
  quiet.word = nullptr;
  // Warpgroup 0 gives registers up here, converged; the epilogue takes them
  // at the top of its branch.
  if constexpr (Cfg::kWideEpi) {
    if (warp < 4) setmaxnreg_dec<Cfg::kRegsLow>();
  }

  if ((warp == 0 || warp == 3) && lane == 0) {
    // ----------------------------------------------- TMA producers (R / X) --
    const bool raw = warp == 0;
    const int depth = raw ? RS : XS;
    uint64_t* full = raw ? r_full : x_full;
    // Swapped layout: an X slot is free when the F slot of the same K block is
    // (same ring depth and order, one commit per stage).
    uint64_t* empty = raw ? r_empty : (kSwap ? f_empty : x_empty);
    int it = 0;  // raw: K blocks; X: X stages of kFKB K blocks
    bool aborted = false;
    for (int t = blockIdx.x; t < num_units && !aborted; t += gridDim.x) {
      const QUnit u = unit_of(t, args);
      for (int kb = u.kb0; kb < u.kb1; kb += raw ? 1 : Cfg::kFKB, ++it) {
        const int s = it % depth;
        const uint32_t ph = (it / depth) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, args.st, raw ? 0x2100 : 0x2101)) { aborted = true; break; }
        if (raw) {
          uint8_t* st = sR + s * Cfg::kRawBytes;
          mbar_arrive_expect_tx(&full[s], Cfg::kRawTx);
#pragma unroll
          for (int g = 0; g < kNT; ++g) {
            uint8_t* sg = st + g * Cfg::kRawTileBytes;
            const int n0 = u.nb * kUnitN + g * kTileN;
            if (kQ == kInt8) {
              tma_load_2d(sg, &tmW, &full[s], n0, kb * kBK);
            } else {
              tma_load_2d(sg, &tmW, &full[s], n0, kb * (kBK / 2));
              if (!Cfg::kGS) tma_load_2d(sg + 4096, &tmS, &full[s], n0, (kb * kBK) / 128);
            }
          }
        } else {
          // Both K blocks of a stage (the second may lie past the unit's K
          // range, or past K where the copy fills zeros; the MMAs skip it).
          mbar_arrive_expect_tx(&full[s], Cfg::kXBytes);
#pragma unroll
          for (int b = 0; b < Cfg::kFKB; ++b) {
            tma_load_2d(sX + s * Cfg::kXBytes + b * Cfg::kXBlockBytes, &tmX, &full[s], (kb + b) * kBK,
                        kSwap ? 0 : u.mb * kNX);
          }
          if (Cfg::kF8Lo) {
            tma_load_2d(sX + s * Cfg::kXBytes + Cfg::kFKB * Cfg::kXBlockBytes, &tmX8, &full[s], kb * kBK, u.mb * kNX);
          }
        }
      }
    }
    if (aborted) {
      for (int i = (it > depth ? it - depth : 0); i < it; ++i) {
        mbar_wait(&full[i % depth], (i / depth) & 1, never_flag, quiet, 0);
      }
    }
  } else if (warp == 1 && (kSwap || lane == 0)) {
    // ---------------------------------------------------------- MMA issuer --
    // Swapped layout: the whole warp runs the loop (warp-uniform state stays
    // in uniform registers, which tcgen05.mma takes its operands from) and one
    // elected lane issues the MMAs and commits; its small N = 16..64 MMAs
    // were issue-bound from a single lane (~90 cycles per MMA, measured; ~30
    // this way). The M >= 65 layout keeps the single-lane loop (measured
    // faster there: its N = 128..256 MMAs are bound by the tensor pipe).
    const bool leader = kSwap ? elect_one() : true;
    auto all_lanes = [](bool v) { return kSwap ? __all_sync(0xffffffffu, v) : v; };
    // normal: A = X [128 m x 64 k] K-major, B = W16 [64 k x 128 n] MN-major
    // swap:   A = W16 as [128 n x 64 k] MN-major, B = X [kNX m x 64 k] K-major
    constexpr uint32_t idesc = kSwap ? idesc_f16_f32(128, kNX, 1, 0) : idesc_f16_f32(128, kUnitN, 0, 1);
    // The issuer's per-stage work bounds the small-M rate: the whole-unit
    // form below keeps its loop minimal; group runs (kGS) add a buffer
    // switch per run.
    if constexpr (Cfg::kGS) {
      int it = 0;
      int tc = 0;  // accumulator runs: one per group run
      bool aborted = false;
      for (int t = blockIdx.x; t < num_units && !aborted; t += gridDim.x) {
        const QUnit u = unit_of(t, args);
        int buf = 0;
        uint32_t d_tmem = tmem;
        for (int kb = u.kb0; kb < u.kb1; kb += Cfg::kFKB, ++it) {
          const int nkb = Cfg::kFKB == 1 ? 1 : min(Cfg::kFKB, u.kb1 - kb);
          const bool first = run_starts(kb, u.kb0);
          if (first) {
            buf = tc % Cfg::kAccBufs;
            const uint32_t use = tc / Cfg::kAccBufs;
            if (!all_lanes(mbar_wait(&acc_empty[buf], (use & 1) ^ 1, abort_flag, args.st, 0x2200))) {
              aborted = true;
              break;
            }
            tc_fence_after();
            d_tmem = tmem + buf * Cfg::kAccCols;
          }
          const int fs = it % FS, xs = it % XS;
          if (!all_lanes(mbar_wait(&f_full[fs], (it / FS) & 1, abort_flag, args.st, 0x2201) &&
                                   mbar_wait(&x_full[xs], (it / XS) & 1, abort_flag, args.st, 0x2202))) {
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint64_t xd0 = sdesc_sw128(smem_u32(sX + xs * Cfg::kXBytes), 16, 1024);
          // F stage = [channel tile g][64 k][128 n] fp16 (then, int4 M >= 129,
          // the E5M2 w_lo tiles): with kNT = 2 one N = 256 instruction covers
          // both tiles (64-channel chunks 8 KB apart throughout).
          const uint64_t wd0 = sdesc_sw128(smem_u32(sF + fs * Cfg::kFBytes), 8192, 1024);
          if (leader) {
#pragma unroll
            for (int kk = 0; kk < Cfg::kFKB * (kBK / 16); ++kk) {
              const int b = kk / (kBK / 16), k = kk % (kBK / 16);
              if (b >= nkb) break;
              const uint64_t xd = xd0 + static_cast<uint64_t>((b * Cfg::kXBlockBytes + k * 32) >> 4);
              const uint64_t wd = wd0 + static_cast<uint64_t>((b * Cfg::kW16BlockBytes + k * 2048) >> 4);
              const uint32_t acc = (!first || kk != 0) ? 1u : 0u;
              if (kSwap) {
#pragma unroll
                for (int g = 0; g < kNT; ++g) {
                  umma_f16_ss(d_tmem + g * kNX, wd + static_cast<uint64_t>((g * Cfg::kW16Bytes) >> 4), xd, idesc, acc);
                }
              } else {
#pragma unroll
                for (int h = 0; h < Cfg::kRowHalves; ++h) {
                  umma_f16_ss(d_tmem + h * kUnitN, xd + static_cast<uint64_t>((h * 16384) >> 4), wd, idesc, acc);
                }
              }
            }
            umma_commit(&f_empty[fs]);
            if (!kSwap) umma_commit(&x_empty[xs]);
            if (run_ends(kb + nkb - 1, u.kb1)) umma_commit(&acc_full[buf]);
          }
          if (kSwap) __syncwarp();
          if (run_ends(kb + nkb - 1, u.kb1)) ++tc;
        }
      }
    } else {
      int it = 0, tc = 0;
      bool aborted = false;
      for (int t = blockIdx.x; t < num_units && !aborted; t += gridDim.x, ++tc) {
        const QUnit u = unit_of(t, args);
        const int buf = tc % Cfg::kAccBufs;
        const uint32_t use = tc / Cfg::kAccBufs;
        if (!all_lanes(mbar_wait(&acc_empty[buf], (use & 1) ^ 1, abort_flag, args.st, 0x2200))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + buf * Cfg::kAccCols;
        for (int kb = u.kb0; kb < u.kb1; kb += Cfg::kFKB, ++it) {
          const int nkb = Cfg::kFKB == 1 ? 1 : min(Cfg::kFKB, u.kb1 - kb);
          const int fs = it % FS, xs = it % XS;
          if (!all_lanes(mbar_wait(&f_full[fs], (it / FS) & 1, abort_flag, args.st, 0x2201) &&
                                   mbar_wait(&x_full[xs], (it / XS) & 1, abort_flag, args.st, 0x2202))) {
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint64_t xd0 = sdesc_sw128(smem_u32(sX + xs * Cfg::kXBytes), 16, 1024);
          // F stage = [channel tile g][64 k][128 n] fp16 (then, int4 M >= 129,
          // the E5M2 w_lo tiles): with kNT = 2 one N = 256 instruction covers
          // both tiles (64-channel chunks 8 KB apart throughout).
          const uint64_t wd0 = sdesc_sw128(smem_u32(sF + fs * Cfg::kFBytes), 8192, 1024);
          if (leader) {
#pragma unroll
            for (int kk = 0; kk < Cfg::kFKB * (kBK / 16); ++kk) {
              const int b = kk / (kBK / 16), k = kk % (kBK / 16);
              if (b >= nkb) break;
              const uint64_t xd = xd0 + static_cast<uint64_t>((b * Cfg::kXBlockBytes + k * 32) >> 4);
              const uint64_t wd = wd0 + static_cast<uint64_t>((b * Cfg::kW16BlockBytes + k * 2048) >> 4);
              const uint32_t acc = (kb != u.kb0 || kk != 0) ? 1u : 0u;
              if (kSwap) {
#pragma unroll
                for (int g = 0; g < kNT; ++g) {
                  umma_f16_ss(d_tmem + g * kNX, wd + static_cast<uint64_t>((g * Cfg::kW16Bytes) >> 4), xd, idesc, acc);
                }
              } else {
#pragma unroll
                for (int h = 0; h < Cfg::kRowHalves; ++h) {
                  umma_f16_ss(d_tmem + h * kUnitN, xd + static_cast<uint64_t>((h * 16384) >> 4), wd, idesc, acc);
                }
              }
            }
            if constexpr (Cfg::kF8Lo) {
              // w_lo: A = E5M2 X (2^-8 x) [rows][64 k] K-major, 64-byte swizzle;
              // B = E5M2 2^8 w_lo [64 k][kUnitN n] MN-major (tiles 8 KB apart).
              // Two K = 32 steps per K block into the same accumulators.
              constexpr uint32_t idesc8 = idesc_e5m2_f32(128, kUnitN, 0, 1);
              const uint64_t x8d = sdesc_sw64(smem_u32(sX + xs * Cfg::kXBytes + Cfg::kFKB * Cfg::kXBlockBytes), 16, 512);
              const uint64_t lod = sdesc_sw128(smem_u32(sF + fs * Cfg::kFBytes + kNT * Cfg::kW16Bytes),
                                               Cfg::kLoBlockBytes, 1024);
#pragma unroll
              for (int k2 = 0; k2 < kBK / 32; ++k2) {
#pragma unroll
                for (int h = 0; h < Cfg::kRowHalves; ++h) {
                  umma_f8_ss(d_tmem + h * kUnitN, x8d + static_cast<uint64_t>((h * 128 * kBK + k2 * 32) >> 4),
                             lod + static_cast<uint64_t>((k2 * 32 * 128) >> 4), idesc8, 1u);
                }
              }
            }
            umma_commit(&f_empty[fs]);
            if (!kSwap) umma_commit(&x_empty[xs]);
          }
          if (kSwap) __syncwarp();
        }
        if (!aborted && leader) umma_commit(&acc_full[buf]);
      }
    }
    if (leader) umma_commit(mma_done);
    if (kSwap) __syncwarp();
    mbar_wait(mma_done, 0, never_flag, quiet, 0);
  } else if (Cfg::kGS && warp == 2 && lane == 0) {
    // ------------------------------------------------ scale rows (int4 TMA) --
    // One row of 128 fp16 scales per weight tile and group run, into a ring
    // the epilogue warps release.
    constexpr int SS = Cfg::kScSlots > 0 ? Cfg::kScSlots : 1;
    int si = 0;
    bool aborted = false;
    for (int t = blockIdx.x; t < num_units && !aborted; t += gridDim.x) {
      const QUnit u = unit_of(t, args);
      for (int kb = u.kb0; kb < u.kb1; ++kb) {
        if (!run_starts(kb, u.kb0)) continue;
        const int slot = si % SS;
        if (!mbar_wait(&sc_empty[slot], ((si / SS) & 1) ^ 1, abort_flag, args.st, 0x2102)) {
          aborted = true;
          break;
        }
        mbar_arrive_expect_tx(&sc_full[slot], Cfg::kScBytes);
#pragma unroll
        for (int g = 0; g < kNT; ++g) {
          tma_load_2d(sSc + slot * Cfg::kScBytes + g * 256, &tmS, &sc_full[slot], u.nb * kUnitN + g * kTileN,
                      (kb * kBK) / 128);
        }
        ++si;
      }
    }
    if (aborted) {
      for (int i = (si > SS ? si - SS : 0); i < si; ++i) mbar_wait(&sc_full[i % SS], (i / SS) & 1, never_flag, quiet, 0);
    }
  } else if ((warp >= 4 && warp < 8) || warp >= 12) {
    // ------------------------------------------------------------- convert --
    // Two convert groups (warps 4-7 and 12-15) take alternate K blocks, so
    // one block is dequantised while the other group's is being stored, and
    // convert all tiles of their block (kGroupTiles). The M >= 65 layout with
    // two weight tiles per unit instead gives each group its own tile (grp)
    // of every K block.
    const int grp = warp >= 12 ? 1 : 0;
    const int ct = threadIdx.x - (grp ? 384 : 128);  // 0..127
    int it = 0;  // F stages
    int ri = 0;  // K blocks: position in the raw ring
    bool ok_run = true;
    for (int t = blockIdx.x; t < num_units && ok_run; t += gridDim.x) {
      const QUnit u = unit_of(t, args);
      for (int kb = u.kb0; kb < u.kb1 && ok_run; kb += Cfg::kFKB, ++it) {
        const int nkb = Cfg::kFKB == 1 ? 1 : min(Cfg::kFKB, u.kb1 - kb);
        if (Cfg::kAltStages && (it & 1) != grp) {
          ri += nkb;
          continue;
        }
        const int fs = it % FS;
        for (int b = 0; b < nkb; ++b, ++ri) {
          const int rs = ri % RS;
          if (!mbar_wait(&r_full[rs], (ri / RS) & 1, abort_flag, args.st, 0x2300)) { ok_run = false; break; }
          constexpr int GT = Cfg::kGroupTiles;
          const uint8_t* raw = sR + rs * Cfg::kRawBytes + (Cfg::kAltStages ? 0 : grp * Cfg::kRawTileBytes);
          uint8_t* w16 = sF + fs * Cfg::kFBytes + b * Cfg::kW16BlockBytes + (Cfg::kAltStages ? 0 : grp * Cfg::kW16Bytes);
          if (kQ == kInt8) {
            // thread -> (k row r, n half h); raw unit u of row r sits at unit u ^ (r & 7).
            // Each group of 8 consecutive threads takes 8 consecutive rows of one
            // half, so its 16-byte accesses fall in 8 different bank groups.
            const int r = (ct & 7) + 8 * (ct >> 4);
            const int h = (ct >> 3) & 1;
            const int sw = r & 7;
            uint4 o[GT][8];
#pragma unroll
            for (int g = 0; g < GT; ++g) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint4 rv = *reinterpret_cast<const uint4*>(raw + g * Cfg::kRawTileBytes + r * 128 +
                                                                 (((4 * h + i) ^ sw) << 4));
                dequant_i8x16(rv, o[g][2 * i], o[g][2 * i + 1]);
              }
            }
            // The raw slot is released only once its bytes have been consumed
            // into registers (the dequantised values depend on them): a release
            // right after issuing the loads lets the next TMA write overtake
            // loads that have not been performed yet.
            __syncwarp();
            if (lane == 0) mbar_arrive(&r_empty[rs]);
            if (b == 0 && !mbar_wait(&f_empty[fs], ((it / FS) & 1) ^ 1, abort_flag, args.st, 0x2301)) {
              ok_run = false;
              break;
            }
#pragma unroll
            for (int g = 0; g < GT; ++g) {
              uint8_t* dst = w16 + g * Cfg::kW16Bytes + h * 8192 + r * 128;
#pragma unroll
              for (int i = 0; i < 8; ++i) *reinterpret_cast<uint4*>(dst + ((i ^ sw) << 4)) = o[g][i];
            }
          } else {
            if constexpr (Cfg::kGS) {
              // thread -> (byte row kk: k rows 2kk and 2kk+1, n quarter qn: 32 channels)
              const int kk = ct >> 2;
              const int qn = ct & 3;
              const int swr = kk & 7;
              const __half2 b8 = __float2half2_rn(1032.f);  // 1024 + 8
              uint32_t hv[GT][2][2][8];  // [tile][raw unit i][row r0/r1][16 channels as 8 half2]
#pragma unroll
              for (int g = 0; g < GT; ++g) {
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                  const uint4 rv = *reinterpret_cast<const uint4*>(raw + g * Cfg::kRawTileBytes + kk * 128 +
                                                                   (((2 * qn + i) ^ swr) << 4));
                  const uint32_t words[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                  for (int wdx = 0; wdx < 4; ++wdx) {
                    const uint32_t lo_n = (words[wdx] & 0x0F0F0F0Fu) ^ 0x08080808u;         // k even
                    const uint32_t hi_n = ((words[wdx] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;  // k odd
#pragma unroll
                    for (int half_sel = 0; half_sel < 2; ++half_sel) {
                      const uint32_t sel = half_sel ? 0x7362u : 0x5140u;
                      hv[g][i][0][wdx * 2 + half_sel] = h2_as_u32(__hsub2(u32_as_h2(bytes_to_h2(lo_n, sel)), b8));
                      hv[g][i][1][wdx * 2 + half_sel] = h2_as_u32(__hsub2(u32_as_h2(bytes_to_h2(hi_n, sel)), b8));
                    }
                  }
                }
              }
              // Release the raw slot only after its bytes are consumed (see int8).
              __syncwarp();
              if (lane == 0) mbar_arrive(&r_empty[rs]);
              if (b == 0 && !mbar_wait(&f_empty[fs], ((it / FS) & 1) ^ 1, abort_flag, args.st, 0x2301)) {
              ok_run = false;
              break;
            }
              const int chunk = qn >> 1;
#pragma unroll
              for (int g = 0; g < GT; ++g) {
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                  // 16 channels = two fp16 units; column within the chunk = 32 (qn & 1) + 16 i
                  const int v0 = 4 * (qn & 1) + 2 * i;
#pragma unroll
                  for (int rr = 0; rr < 2; ++rr) {
                    const int row = 2 * kk + rr;
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                      const int off = g * Cfg::kW16Bytes + chunk * 8192 + row * 128 + (((v0 + e) ^ (row & 7)) << 4);
                      *reinterpret_cast<uint4*>(w16 + off) =
                          make_uint4(hv[g][i][rr][4 * e], hv[g][i][rr][4 * e + 1], hv[g][i][rr][4 * e + 2],
                                     hv[g][i][rr][4 * e + 3]);
                    }
                  }
                }
              }
            } else {
              // thread -> (byte row kk: k rows 2kk and 2kk+1, n quarter qn: 32 channels)
              const int kk = ct >> 2;
              const int qn = ct & 3;
              const int swr = kk & 7;
              const __half* sc = reinterpret_cast<const __half*>(raw + 4096) + qn * 32;
              const __half2 b8 = __float2half2_rn(1032.f);  // 1024 + 8
              const __half2 h256 = __float2half2_rn(256.f);
              uint32_t hv[2][2][8], lv[2][2][8];  // [raw unit i][row r0/r1][16 channels as 8 half2]
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                const uint4 rv = *reinterpret_cast<const uint4*>(raw + kk * 128 + (((2 * qn + i) ^ swr) << 4));
                const uint32_t words[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                for (int wdx = 0; wdx < 4; ++wdx) {
                  const uint32_t lo_n = (words[wdx] & 0x0F0F0F0Fu) ^ 0x08080808u;         // k even
                  const uint32_t hi_n = ((words[wdx] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;  // k odd
#pragma unroll
                  for (int half_sel = 0; half_sel < 2; ++half_sel) {
                    const uint32_t sel = half_sel ? 0x7362u : 0x5140u;
                    const __half2 s2 = *reinterpret_cast<const __half2*>(sc + 16 * i + 4 * wdx + 2 * half_sel);
                    const __half2 q0 = __hsub2(u32_as_h2(bytes_to_h2(lo_n, sel)), b8);
                    const __half2 q1 = __hsub2(u32_as_h2(bytes_to_h2(hi_n, sel)), b8);
                    const __half2 w0h = __hmul2(q0, s2);
                    const __half2 w1h = __hmul2(q1, s2);
                    // w_lo = q * s - w_hi (exact in fp16), times 2^8 (exact)
                    hv[i][0][wdx * 2 + half_sel] = h2_as_u32(w0h);
                    lv[i][0][wdx * 2 + half_sel] = h2_as_u32(__hmul2(__hfma2(q0, s2, __hneg2(w0h)), h256));
                    hv[i][1][wdx * 2 + half_sel] = h2_as_u32(w1h);
                    lv[i][1][wdx * 2 + half_sel] = h2_as_u32(__hmul2(__hfma2(q1, s2, __hneg2(w1h)), h256));
                  }
                }
              }
              // Release the raw slot only after its bytes are consumed (see int8).
              __syncwarp();
              if (lane == 0) mbar_arrive(&r_empty[rs]);
              if (b == 0 && !mbar_wait(&f_empty[fs], ((it / FS) & 1) ^ 1, abort_flag, args.st, 0x2301)) {
              ok_run = false;
              break;
            }
              uint8_t* hi = w16;
              // E5M2 w_lo of this tile: [64 k][128 n] bytes, 128-byte swizzle.
              uint8_t* lo8 = sF + fs * Cfg::kFBytes + kNT * Cfg::kW16Bytes +
                             (Cfg::kAltStages ? 0 : grp * Cfg::kLoBlockBytes);
              const int chunk = qn >> 1;
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                // 16 channels = two fp16 units; column within the chunk = 32 (qn & 1) + 16 i
                const int v0 = 4 * (qn & 1) + 2 * i;
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                  const int row = 2 * kk + rr;
#pragma unroll
                  for (int e = 0; e < 2; ++e) {
                    const int off = chunk * 8192 + row * 128 + (((v0 + e) ^ (row & 7)) << 4);
                    *reinterpret_cast<uint4*>(hi + off) = make_uint4(hv[i][rr][4 * e], hv[i][rr][4 * e + 1],
                                                                     hv[i][rr][4 * e + 2], hv[i][rr][4 * e + 3]);
                  }
                  // 2^8 w_lo has at most 3 significant bits: as a normal fp16
                  // its low byte is zero and its high byte is the E5M2 value.
                  uint32_t w8[4];
#pragma unroll
                  for (int j = 0; j < 4; ++j) w8[j] = __byte_perm(lv[i][rr][2 * j], lv[i][rr][2 * j + 1], 0x7531);
                  *reinterpret_cast<uint4*>(lo8 + row * 128 + (((2 * qn + i) ^ (row & 7)) << 4)) =
                      make_uint4(w8[0], w8[1], w8[2], w8[3]);
                }
              }
            }
          }
        }
        if (!ok_run) break;
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&f_full[fs]);
      }
    }
  } else if (warp >= 8 && warp < 12) {
    // ------------------------------------------------------------ epilogue --
    if constexpr (Cfg::kWideEpi) setmaxnreg_inc<Cfg::kRegsEpi>();
    const uint32_t q = warp & 3;
    const int lrow = q * 32 + lane;  // TMEM lane: m (normal) or n (swap)
    const uint32_t lane_base = tmem + ((q * 32) << 16);
    if constexpr (Cfg::kGS) {
      // Running sums in registers: += group-run partial * fp32(scale[g][n]);
      // lane = channel, kNT tiles x kNX rows of X.
      constexpr int SS = Cfg::kScSlots;
      constexpr int NC = kNT * kNX;
      int tc = 0, si = 0;
      bool ok_run = true;
      for (int t = blockIdx.x; t < num_units && ok_run; t += gridDim.x) {
        const QUnit u = unit_of(t, args);
        float accv[NC];
#pragma unroll
        for (int i = 0; i < NC; ++i) accv[i] = 0.f;
        for (int kb = u.kb0; kb < u.kb1; ++kb) {
          if (!run_ends(kb, u.kb1)) continue;
          const int buf = tc & 1;
          const int slot = si % SS;
          const bool got = mbar_wait(&acc_full[buf], (tc >> 1) & 1, abort_flag, args.st, 0x2400) &&
                           mbar_wait(&sc_full[slot], (si / SS) & 1, abort_flag, args.st, 0x2401);
          if (!__all_sync(0xffffffffu, got)) {
            ok_run = false;
            break;
          }
          tc_fence_after();
          const uint32_t acc = lane_base + buf * Cfg::kAccCols;
          const __half* scr = reinterpret_cast<const __half*>(sSc + slot * Cfg::kScBytes);
#pragma unroll
          for (int g = 0; g < kNT; ++g) {
            const float sc = __half2float(scr[g * kTileN + lrow]);
#pragma unroll
            for (int c = 0; c < (kNX + 31) / 32; ++c) {
              uint32_t r[32];
              if constexpr (kNX >= 32) {
                tmem_ld32(acc + g * kNX + c * 32, r);
              } else {
                uint32_t r16[16];
                tmem_ld16(acc + g * kNX, r16);
#pragma unroll
                for (int i = 0; i < 16; ++i) r[i] = r16[i];
              }
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < (kNX >= 32 ? 32 : kNX); ++i) {
                accv[g * kNX + c * 32 + i] = fmaf(__uint_as_float(r[i]), sc, accv[g * kNX + c * 32 + i]);
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&acc_empty[buf]);
            mbar_arrive(&sc_empty[slot]);
          }
          ++tc;
          ++si;
        }
        if (!ok_run) break;
        // The unit's sums -> Y, or this K split's partial sums.
        float* ydst = args.partial != nullptr ? args.partial + static_cast<int64_t>(u.ks) * args.M * args.N : args.Y;
        const int64_t ld = args.partial != nullptr ? args.N : args.ldy;
#pragma unroll
        for (int g = 0; g < kNT; ++g) {
          const int n = u.nb * kUnitN + g * kTileN + lrow;
          if (n < args.N) {
#pragma unroll
            for (int m = 0; m < kNX; ++m) {
              if (m < args.M) ydst[static_cast<int64_t>(m) * ld + n] = accv[g * kNX + m];
            }
          }
        }
      }
    } else {
    int tc = 0;
    int y_commits = 0;  // TMA stores this warp committed (staging block parity)
    for (int t = blockIdx.x; t < num_units; t += gridDim.x, ++tc) {
      const QUnit u = unit_of(t, args);
      const int mb = u.mb;
      const int nb = u.nb;
      // split-K: raw partial sums (no scale) go to partial[ks]; the reduce
      // kernel applies the scale. Otherwise straight to Y.
      float* ydst = args.partial != nullptr ? args.partial + static_cast<int64_t>(u.ks) * args.M * args.N : args.Y;
      const int64_t ld = args.partial != nullptr ? args.N : args.ldy;
      const __half* csc = args.partial != nullptr ? nullptr : args.chan_scale;
      const float* tsc = args.partial != nullptr ? nullptr : args.tensor_scale;
      const int buf = tc % Cfg::kAccBufs;
      const uint32_t use = tc / Cfg::kAccBufs;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], use & 1, abort_flag, args.st, 0x2400))) break;
      tc_fence_after();
      const uint32_t acc = lane_base + buf * Cfg::kAccCols;
      if (kSwap) {
#pragma unroll 1
        for (int g = 0; g < kNT; ++g) {
          const int n = nb * kUnitN + g * kTileN + lrow;
          const float sc = (csc != nullptr && n < args.N) ? __half2float(csc[n])
                                                          : (tsc != nullptr ? __ldg(tsc) : 1.f);
#pragma unroll
          for (int c = 0; c < (kNX + 31) / 32; ++c) {
            uint32_t r[32];
            if (kNX >= 32) {
              tmem_ld32(acc + g * kNX + c * 32, r);
            } else {
              uint32_t r16[16];
              tmem_ld16(acc + g * kNX, r16);
#pragma unroll
              for (int i = 0; i < 16; ++i) r[i] = r16[i];
            }
            tmem_wait_ld();
            if (n < args.N) {
#pragma unroll
              for (int i = 0; i < (kNX >= 32 ? 32 : kNX); ++i) {
                const int m = c * 32 + i;
                if (m < args.M) ydst[static_cast<int64_t>(m) * ld + n] = __uint_as_float(r[i]) * sc;
              }
            }
          }
        }
      } else if (args.y_tma) {
        // Rows of 32 channels through 128-byte-swizzled staging (16 rows at a
        // time) and TMA stores: full-line writes instead of one 4-byte store
        // per row and channel, which left the L1 busy with the epilogue.
        uint8_t* stage0 = smem + Cfg::kOffOut + (warp - 8) * 2048 * Cfg::kOutBufs;
#pragma unroll 1
        for (int hc = 0; hc < Cfg::kRowHalves * (kUnitN / 32); ++hc) {
          const int h = hc / (kUnitN / 32), c = hc % (kUnitN / 32);
          const int m0 = mb * kNX + h * 128 + static_cast<int>(q) * 32;
          uint32_t r[32];
          tmem_ld32(acc + h * kUnitN + c * 32, r);
          tmem_wait_ld();
          const int n0 = nb * kUnitN + c * 32;
          if (csc != nullptr) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float sc = n0 + i < args.N ? __half2float(__ldg(csc + n0 + i)) : 0.f;
              r[i] = __float_as_uint(__uint_as_float(r[i]) * sc);
            }
          } else if (tsc != nullptr) {
            const float sc = __ldg(tsc);
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * sc);
          }
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            // Two blocks: write the one the latest committed store did not
            // use, once every older store has read its block.
            uint8_t* stage = stage0 + (Cfg::kOutBufs == 2 ? (y_commits & 1) * 2048 : 0);
            if (lane == 0) {
              if (Cfg::kOutBufs == 2) {
                bulk_wait_read_but1();
              } else {
                bulk_wait_read_all();
              }
            }
            __syncwarp();
            if ((lane >> 4) == static_cast<uint32_t>(half)) {
              const uint32_t row = lane & 15;
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                *reinterpret_cast<uint4*>(stage + row * 128 + ((v ^ (row & 7)) << 4)) =
                    make_uint4(r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
              }
            }
            fence_async_smem();
            __syncwarp();
            if (m0 + 16 * half < args.M && n0 < args.N) {  // warp-uniform
              if (lane == 0) {
                tma_store_3d(&tmY, stage, n0, m0 + 16 * half, args.partial != nullptr ? u.ks : 0);
                bulk_commit();
              }
              ++y_commits;
            }
          }
        }
      } else {
#pragma unroll 1
        for (int hc = 0; hc < Cfg::kRowHalves * (kUnitN / 32); ++hc) {
          const int h = hc / (kUnitN / 32), c = hc % (kUnitN / 32);
          const int m = mb * kNX + h * 128 + lrow;
          float* yrow = ydst + static_cast<int64_t>(m) * ld;
          uint32_t r[32];
          tmem_ld32(acc + h * kUnitN + c * 32, r);
          tmem_wait_ld();
          const int n0 = nb * kUnitN + c * 32;
          if (m < args.M) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int n = n0 + i;
              if (n < args.N) {
                const float sc = csc != nullptr ? __half2float(__ldg(csc + n)) : (tsc != nullptr ? __ldg(tsc) : 1.f);
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
    if (lane == 0) bulk_wait_all();  // this warp's Y stores are complete before the CTA exits
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
  const float* tscale = nullptr;  // int8 only: one fp32 scale for all of Y (when `scale` is null)
  float* Y;
  int64_t ldy;
  int M, N, K;
  int kind;
  // split-K plan (filled by plan_splits) and the fp32 partial-sum buffer
  int splits = 1;
  int kb_per_split = 0;
  int pair = 0;   // two 128-channel tiles per unit (M >= 65 layout, and M <= 16)
  int rows2 = 0;  // units of 256 rows (two accumulators): W8A16 paired, W4A16 single
  float* partial = nullptr;
  DevStatus st{};
};

// M >= 65 layout: choose the unit shape and a K split from a cost model in
// units of one 128 x 128, whole-K unit: waves x unit cost x share of K, plus
// the split-K cost (a reduce launch and the partial sums' write and read, at
// HBM speed). Measured on B200 (K = 4096, N = 11008) relative to a single
// unit: 128 rows x 256 channels (paired tiles) 1.31-1.42x (int8) / 1.82x
// (int4); 256 x 256 (W8A16) 1.9-2.0x; 256 x 128 (W4A16) 1.4x; a single unit
// streams a 64-deep K block in about 0.6 us. Split plans whose partial sums exceed max_partial
// floats are not considered.
void plan_normal(QProblem& p, int sms, size_t max_partial) {
  const int num_k = (p.K + kBK - 1) / kBK;
  const double unit_us = 0.6 * num_k;
  // K splits only when even single tiles leave most SMs idle (measured: they
  // help W8A16 at M = 65..128, N = 11008, and lose once the tiles fill a
  // wave; W4A16 measured no gain at M = 128).
  const int64_t single_units = static_cast<int64_t>((p.M + 127) / 128) * ((p.N + kTileN - 1) / kTileN);
  const int max_sp = (p.kind == kInt8 && single_units < static_cast<int64_t>(0.6 * sms)) ? 4 : 1;
  // 256-row units keep Y whole-tile TMA stores (aligned Y) and no K split.
  const bool rows2_ok = p.M > 128 && p.ldy % 4 == 0 && (reinterpret_cast<uintptr_t>(p.Y) & 15u) == 0;
  const bool w8 = p.kind == kInt8;
  struct Shape { int rows, chans, pair, rows2; double cost; bool ok; };
  const Shape shapes[4] = {{128, 128, 0, 0, 1.0, true},
                           {128, 256, 1, 0, w8 ? 1.35 : 1.85, true},
                           {256, 256, 1, 1, 1.95, w8},
                           {256, 128, 0, 1, 1.42, !w8}};
  double best = 1e30;
  for (const Shape& sh : shapes) {
    if (!sh.ok || (sh.rows2 && !rows2_ok)) continue;
    const int64_t base = static_cast<int64_t>((p.M + sh.rows - 1) / sh.rows) * ((p.N + sh.chans - 1) / sh.chans);
    for (int sp = 1; sp <= (sh.rows2 ? 1 : max_sp) && sp <= num_k; ++sp) {
      const int kbps = (num_k + sp - 1) / sp;
      const int real = (num_k + kbps - 1) / kbps;
      if (sp > 1 && real == 1) continue;
      if (real > 1 && static_cast<size_t>(real) * p.M * p.N > max_partial) continue;
      if (real > 1 && p.N % 4 != 0) continue;  // partial rows must suit TMA stores
      const int64_t waves = (base * real + sms - 1) / sms;
      double t = static_cast<double>(waves) * sh.cost * kbps / num_k;
      if (real > 1) t += (3.0 + real * 8.0 * p.M * p.N / 5e6) / unit_us;
      if (t < best * 0.98) {
        best = t;
        p.pair = sh.pair;
        p.rows2 = sh.rows2;
        p.splits = real;
        p.kb_per_split = kbps;
      }
    }
  }
}

// Split K when the output tiles alone cannot fill the SMs (small M): pick the
// split count whose units fill the persistent grid best, preferring fewer
// splits (each split adds an M x N fp32 partial write and read).
// Operands swapped (W as the 128-row A operand, X as B with N' = M): M <= 64,
// and int4 up to M = 128 (its group-scaled sums keep the weights exact in one
// fp16 MMA per K step; the M >= 65 layout leaves SMs idle at M = 128).
bool swapped_layout(const QProblem& p) { return p.M <= 64 || (p.kind == kInt4G128 && p.M <= 128); }

void plan_splits(QProblem& p, int sms, size_t max_partial = SIZE_MAX) {
  const bool swap = swapped_layout(p);
  const int num_m = swap ? 1 : (p.M + 127) / 128;
  const int num_k = (p.K + kBK - 1) / kBK;
  p.splits = 1;
  p.kb_per_split = num_k;
  p.pair = 0;
  p.rows2 = 0;
  if (!swap) {
    plan_normal(p, sms, max_partial);
    return;
  }
  // M <= 16: two 128-channel tiles per unit (both convert groups on every K
  // block, two MMAs per K step): W8A16 M=16 31 -> 27 us; no gain from M = 32.
  // (Not in the allocation-free entry, whose split plans keep the single-tile
  // unit count its fixed scratch was sized for.)
  p.pair = (p.M <= 16 && max_partial == SIZE_MAX) ? 1 : 0;
  const int sbase = num_m * ((p.N + (kTileN << p.pair) - 1) / (kTileN << p.pair));
  if (sbase >= sms || num_k < 2) return;
  // Each split writes and re-reads an M x N fp32 partial: keep that traffic
  // under a tenth of the weight stream, or let the partials take up to 48 MB
  // (they stay in L2; measured faster for M = 16).
  const double wbytes = (p.kind == kInt8 ? 1.0 : 0.5) * static_cast<double>(p.K) * p.N;
  const double per_split = 4.0 * p.M * p.N;
  const int max_splits = static_cast<int>(std::max(0.1 * wbytes / (2.0 * per_split), 48e6 / per_split));
  if (max_splits < 2) return;
  double best = static_cast<double>(sbase) / sms;
  for (int sp = 2; sp <= 16 && sp <= num_k && sp <= max_splits; ++sp) {
    int kbps = (num_k + sp - 1) / sp;
    if (p.kind == kInt4G128 || p.pair) kbps += kbps & 1;  // splits start on a two-block stage boundary
    const int real = (num_k + kbps - 1) / kbps;  // no empty split
    if (static_cast<size_t>(real) * p.M * p.N > max_partial) continue;  // partial sums must fit the scratch
    const int64_t units = static_cast<int64_t>(sbase) * real;
    const int64_t waves = (units + sms - 1) / sms;
    const double eff = static_cast<double>(units) / static_cast<double>(waves * sms) * (1.0 - 0.01 * real);
    if (eff > best + 0.02) {
      best = eff;
      p.splits = real;
      p.kb_per_split = kbps;
    }
  }
}

// Y[m, n] = scale[n] * sum_s partial[s][m][n] (or tscale[0] * ...), fixed
// summation order.
// Y = scale * sum over the K splits of the partial sums, added in split order.
// Every split's value is requested before any is added (one round trip to
// L2 instead of one per split); four consecutive outputs per thread when N
// and the output rows allow 16-byte accesses.
constexpr int kReduceMaxSplits = 16;
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N,
                                     const __half* __restrict__ scale, const float* __restrict__ tscale,
                                     float* __restrict__ Y, int64_t ldy, int vec4) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = static_cast<int64_t>(M) * N;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const float ts = tscale != nullptr ? __ldg(tscale) : 1.f;
  if (vec4) {
    for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < total / 4; q += stride) {
      float4 v[kReduceMaxSplits];
#pragma unroll
      for (int sp = 0; sp < kReduceMaxSplits; ++sp) {
        v[sp] = sp < splits ? __ldcg(reinterpret_cast<const float4*>(partial + sp * total) + q)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int sp = 0; sp < kReduceMaxSplits; ++sp) {
        if (sp < splits) {
          acc.x += v[sp].x;
          acc.y += v[sp].y;
          acc.z += v[sp].z;
          acc.w += v[sp].w;
        }
      }
      const int64_t i = 4 * q;
      const int n = static_cast<int>(i % N);
      if (scale != nullptr) {
        acc.x *= __half2float(scale[n]);
        acc.y *= __half2float(scale[n + 1]);
        acc.z *= __half2float(scale[n + 2]);
        acc.w *= __half2float(scale[n + 3]);
      } else if (tscale != nullptr) {
        acc.x *= ts;
        acc.y *= ts;
        acc.z *= ts;
        acc.w *= ts;
      }
      *reinterpret_cast<float4*>(Y + (i / N) * ldy + n) = acc;
    }
    return;
  }
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total; i += stride) {
    float v[kReduceMaxSplits];
#pragma unroll
    for (int sp = 0; sp < kReduceMaxSplits; ++sp) v[sp] = sp < splits ? __ldcg(partial + sp * total + i) : 0.f;
    float acc = 0.f;
#pragma unroll
    for (int sp = 0; sp < kReduceMaxSplits; ++sp) {
      if (sp < splits) acc += v[sp];
    }
    const int n = static_cast<int>(i % N);
    if (scale != nullptr) {
      acc *= __half2float(scale[n]);
    } else if (tscale != nullptr) {
      acc *= ts;
    }
    Y[(i / N) * ldy + n] = acc;
  }
}

// X8[m][k] = E5M2(2^-8 * X[m][k]) for the w_lo MMAs of int4 in the M >= 65 layout (M >= 129),
// round to nearest, saturating (rows of K bytes). Eight values per thread.
__global__ void x_to_e5m2_kernel(const __half* __restrict__ X, int64_t ldx, int M, int K, uint8_t* __restrict__ X8) {
  pdl_launch_dependents();
  pdl_wait();
  const int per_row = K / 8;
  const int64_t total = static_cast<int64_t>(M) * per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / per_row;
    const int k = static_cast<int>(i % per_row) * 8;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(X + m * ldx + k));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint16_t b[2];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const float2 f = __half22float2(u32_as_h2(w[2 * j + t]));
        // cvt.rn.satfinite.e5m2x2.f32 d, a, b: a -> high byte, b -> low byte
        asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(b[t]) : "f"(f.y * 0.00390625f), "f"(f.x * 0.00390625f));
      }
      o[j] = static_cast<uint32_t>(b[0]) | (static_cast<uint32_t>(b[1]) << 16);
    }
    *reinterpret_cast<uint2*>(X8 + m * K + k) = make_uint2(o[0], o[1]);
  }
}

template <int kQ, bool kSwap, int kNX, int kNT = 1>
int launch_wq(const QProblem& p, cudaStream_t stream) {
  using Cfg = QCfg<kQ, kSwap, kNX, kNT>;
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
  // Y (or the split partial sums [splits][M][N]) as a 3-D tensor for TMA
  // stores of 16 rows x 32 channels.
  CUtensorMap tmY = tmX;
  int y_tma = 0;
  const bool split_out = p.splits > 1;
  float* ybase = split_out ? p.partial : p.Y;
  const int64_t yld = split_out ? p.N : p.ldy;
  if (!kSwap && yld % 4 == 0 && (reinterpret_cast<uintptr_t>(ybase) & 15u) == 0) {
    uint64_t dims[3] = {static_cast<uint64_t>(p.N), static_cast<uint64_t>(p.M), static_cast<uint64_t>(p.splits)};
    uint64_t strides[2] = {static_cast<uint64_t>(yld) * 4, static_cast<uint64_t>(yld) * 4 * p.M};
    uint32_t box[3] = {32, 16, 1};
    int rc = encode_tmap(&tmY, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, ybase, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NESO_OK) return rc;
    y_tma = 1;
  }
  // int4 M >= 129: the E5M2 copy of X for the w_lo MMAs, in the stream's
  // input workspace, written by a conversion kernel launched just before.
  CUtensorMap tmX8 = tmX;
  uint8_t* x8 = nullptr;
  if constexpr (Cfg::kF8Lo) {
    void* ws = nullptr;
    int rc = stream_workspace(stream, static_cast<size_t>(p.M) * p.K, &ws, kWorkspaceInputs);
    if (rc != NESO_OK) return rc;
    x8 = static_cast<uint8_t*>(ws);
    uint64_t dims[2] = {static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.M)};
    uint64_t strides[1] = {static_cast<uint64_t>(p.K)};
    uint32_t box[2] = {64, static_cast<uint32_t>(kNX)};
    rc = encode_tmap(&tmX8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, x8, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc != NESO_OK) return rc;
    if ((reinterpret_cast<uintptr_t>(p.X) & 15u) != 0) return fail(NESO_ERR_MISALIGNED, "activations must be 16-byte aligned");
  }
  QArgs args{};
  args.y_tma = y_tma;
  args.Y = p.Y;
  args.ldy = p.ldy;
  args.chan_scale = kQ == kInt8 ? static_cast<const __half*>(p.scale) : nullptr;
  args.tensor_scale = kQ == kInt8 ? p.tscale : nullptr;
  args.partial = p.splits > 1 ? p.partial : nullptr;
  args.M = p.M;
  args.N = p.N;
  args.K = p.K;
  args.num_m = kSwap ? 1 : (p.M + kNX - 1) / kNX;
  args.num_n = (p.N + kNT * kTileN - 1) / (kNT * kTileN);
  args.num_k = (p.K + kBK - 1) / kBK;
  args.splits = p.splits;
  args.kb_per_split = p.kb_per_split;
  args.st = p.st;
  const int units = args.num_m * args.num_n * args.splits;
  const int grid = units < sm_count() ? units : sm_count();
  auto kern = wq_gemm_kernel<kQ, kSwap, kNX, kNT>;
  {
    cudaFuncAttributes fa{};
    int src = kernel_setup(reinterpret_cast<const void*>(kern), Cfg::kSmemBytes, &fa);
    if (src != NESO_OK) return src;
    // setmaxnreg.inc draws on the block's launch pool: refuse a split it cannot fund.
    if (Cfg::kWideEpi && fa.numRegs < 128) {
      return fail(NESO_ERR_LAUNCH, "wq_gemm: %d registers/thread cannot fund the %u/%u warpgroup split", fa.numRegs,
                  Cfg::kRegsLow, Cfg::kRegsEpi);
    }
  }
  cudaError_t e = cudaSuccess;
  if constexpr (Cfg::kF8Lo) {
    const int64_t items = static_cast<int64_t>(p.M) * (p.K / 8);
    const int blocks = static_cast<int>(std::min<int64_t>((items + 255) / 256, 8 * sm_count()));
    e = launch_pdl(x_to_e5m2_kernel, dim3(blocks), dim3(256), 0, stream, static_cast<const __half*>(p.X),
                   static_cast<int64_t>(p.ldx), p.M, p.K, x8);
    if (e != cudaSuccess) return cuda_fail(e, "X conversion launch");
  }
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), Cfg::kSmemBytes, stream, tmX, tmW, tmS, tmY, tmX8, args);
  if (e != cudaSuccess) return cuda_fail(e, "wq_gemm launch");
  if (args.partial != nullptr) {
    if (args.splits > kReduceMaxSplits) return fail(NESO_ERR_UNSUPPORTED, "split-K plan of %d splits", args.splits);
    const int64_t total = static_cast<int64_t>(p.M) * p.N;
    const int vec4 = (p.N % 4 == 0 && p.ldy % 4 == 0 && (reinterpret_cast<uintptr_t>(p.Y) & 15u) == 0) ? 1 : 0;
    const int64_t items = vec4 ? total / 4 : total;
    const int blocks = static_cast<int>(std::min<int64_t>((items + 255) / 256, 4 * sm_count()));
    // Launched with programmatic serialization: its CTAs are scheduled as the
    // matmul's CTAs exit and wait there for the partial sums.
    e = launch_pdl(splitk_reduce_kernel, dim3(blocks), dim3(256), 0, stream, args.partial, args.splits, p.M, p.N,
                   args.chan_scale, args.tensor_scale, p.Y, p.ldy, vec4);
    if (e != cudaSuccess) return cuda_fail(e, "split-K reduce launch");
  }
  return ok();
}

// ------------------------------------------------------- small-M GEMV path --
// For M <= 4 (int8) or M <= 2 (int4) the tensor-core path spends its time in
// the hand-offs between the weight ring, the dequant warps and the MMAs; the
// work per weight byte is a handful of multiply-adds. This path reads W
// straight from HBM with 16-byte streaming loads (lane = 16 channels of one
// stored row: one k for int8, two k for packed int4), converts in registers
// and accumulates M dot products per channel in fp32. A CTA covers 512
// channels x one slice of K (one wave of CTAs); its warps split the
// slice and reduce through shared memory; the last CTA of a channel block to
// finish adds the slices in a fixed order (deterministic) and writes Y.
// Weights become exact fp16 values two at a time and are multiplied by the
// fp16 activations with Blackwell's mixed-precision fma.rn.f32.f16 (fp16 x
// fp16 product, exact in fp32, added to the fp32 sum with one rounding: the
// same result as converting both to fp32 first).
//   int8: half2 bits 0x64xx | (b ^ 0x80) hold 1024 + b + 128 exactly (one
//         byte permute per two weights), minus 1152 (one f16x2 subtract);
//         the per-channel scale multiplies the final sum (as the reference's
//         scaled kernel applies it in the epilogue, tests/test_quantized_matmul.py:250-260).
//   int4: nibbles q ^ 8 = q + 8 masked into 0x6400 | n (1024 + q + 8, minus
//         1032) or 0x6400 | 16 n (times 1/16, minus 72: both exact); each warp
//         multiplies a 128-wide group's sums by the group's scale when the
//         group ends.
constexpr int kGvChanPerLane = 16;
constexpr int kGvChannels = 32 * kGvChanPerLane;  // 512 per CTA
constexpr int kGvWarpStride = 32 * 17;            // reduction row per warp, padded (bank-conflict free)

template <int kQ, int kM>
struct GvCfg {
  // 16 warps per CTA. int8 M = 1 needs 64 registers per thread, so two CTAs
  // share an SM and one CTA's prologue and final sums overlap the other's
  // weight stream (measured W8A16 M=1 17.3 -> 16.5 us against one CTA of 32
  // warps); the other cases take up to 128 registers, one CTA per SM.
  static constexpr int kThreads = 512;
  static constexpr int kCtasPerSm = (kQ == kInt8 && kM == 1) ? 2 : 1;
  static constexpr int kWarps = kThreads / 32;
  static constexpr int kSmemBytes = kWarps * kGvWarpStride * 4;
};

struct GvArgs {
  const __half* X;
  int64_t ldx;
  const uint8_t* W;
  int64_t ldw;          // bytes per stored row (int8: per k; int4: per pair of k)
  const __half* scale;  // int8: [N] per channel (nullable); int4: [K/128][lds]
  int64_t lds;
  const float* tscale;  // int8: one fp32 scale for all of Y (nullable; exclusive with scale)
  float* Y;
  int64_t ldy;
  float* partial;  // [slices][M][N] when there is more than one slice
  int* counters;   // one per channel block, zero between launches
  int M, N;
  int rows;            // stored rows (int8: K, int4: K / 2)
  int rows_per_slice;  // stored rows per CTA (a multiple of 4 x warps)
};

__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// acc + x * (low or high fp16 half of w2), product exact, one fp32 rounding.
__device__ __forceinline__ float fma_h_lo(uint16_t x, uint32_t w2, float acc) {
  float d;
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tfma.rn.f32.f16 %0, %1, l, %3;\n\t}"
      : "=f"(d) : "h"(x), "r"(w2), "f"(acc));
  return d;
}
__device__ __forceinline__ float fma_h_hi(uint16_t x, uint32_t w2, float acc) {
  float d;
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tfma.rn.f32.f16 %0, %1, h, %3;\n\t}"
      : "=f"(d) : "h"(x), "r"(w2), "f"(acc));
  return d;
}

template <int kQ, int kM>
__global__ void __launch_bounds__(GvCfg<kQ, kM>::kThreads, GvCfg<kQ, kM>::kCtasPerSm) wq_gemv_kernel(GvArgs a) {
  using Cfg = GvCfg<kQ, kM>;
  constexpr int CPL = kGvChanPerLane;
  constexpr int NW = Cfg::kWarps;
  constexpr int U = 4;                      // stored rows per batch; two batches in flight per lane
  constexpr int KPR = kQ == kInt8 ? 1 : 2;  // k per stored row
  extern __shared__ float gsm[];  // the slice of X as fp16, later [NW][kGvWarpStride] partial sums
  __shared__ int is_last;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cb = blockIdx.x;
  const int sl = blockIdx.y;
  const int slices = gridDim.y;
  const int n0 = cb * kGvChannels + lane * CPL;
  const bool active = n0 < a.N;  // the host guarantees N % 16 == 0
  const int r0 = sl * a.rows_per_slice;
  const int r1 = min(r0 + a.rows_per_slice, a.rows);
  const int per_warp = a.rows_per_slice / NW;  // a multiple of U
  const int wr0 = r0 + warp * per_warp;
  const int wr1 = min(wr0 + per_warp, r1);

  // This CTA's weight rows start towards L2 while the previous kernel on the
  // stream finishes (a prefetch reads nothing into the CTA).
  for (int r = r0 + static_cast<int>(threadIdx.x); r < r1; r += Cfg::kThreads) {
    bulk_prefetch_l2(a.W + static_cast<int64_t>(r) * a.ldw + cb * kGvChannels,
                     static_cast<uint32_t>(min(kGvChannels, a.N - cb * kGvChannels)));
  }
  // Launched with programmatic serialization: the next kernel's CTAs may take
  // SM slots as this grid's CTAs exit; nothing global is read or written
  // before the previous kernel on the stream has completed.
  pdl_launch_dependents();
  pdl_wait();

  // The slice of X (k in [KPR r0, KPR r1)) as fp16 bits in shared memory.
  uint16_t* xs = reinterpret_cast<uint16_t*>(gsm);  // [kM][KPR * rows_per_slice]
  const int kspan = KPR * a.rows_per_slice;
  const uint16_t* xg = reinterpret_cast<const uint16_t*>(a.X);
  for (int i = threadIdx.x; i < kM * kspan; i += Cfg::kThreads) {
    const int m = i / kspan, k = KPR * r0 + (i % kspan);
    xs[i] = (m < a.M && k < KPR * r1) ? xg[static_cast<int64_t>(m) * a.ldx + k] : uint16_t(0);
  }
  __syncthreads();

  float acc[kM][CPL];   // int8: the sums; int4: the current group's sums
  float tot[kM][CPL];   // int4: scaled sums of finished groups
#pragma unroll
  for (int m = 0; m < kM; ++m)
#pragma unroll
    for (int i = 0; i < CPL; ++i) acc[m][i] = tot[m][i] = 0.f;

  if (active) {
    const uint8_t* wp = a.W + n0;
    auto load = [&](uint4* dst, int r) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        dst[u] = (r + u < wr1) ? __ldcs(reinterpret_cast<const uint4*>(wp + static_cast<int64_t>(r + u) * a.ldw))
                               : make_uint4(0u, 0u, 0u, 0u);
      }
    };
    uint4 cur[U], nxt[U];
    if (wr0 < wr1) load(cur, wr0);
    for (int r = wr0; r < wr1; r += U) {
      if (r + U < wr1) load(nxt, r + U);  // next batch in flight while this one is used
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const bool row_ok = r + u < wr1;
        const int kl = KPR * (r + u - r0);  // k index within the slice
        const uint32_t words[4] = {cur[u].x, cur[u].y, cur[u].z, cur[u].w};
        if (kQ == kInt8) {
          uint16_t xv[kM];
#pragma unroll
          for (int m = 0; m < kM; ++m) xv[m] = row_ok ? xs[m * kspan + kl] : uint16_t(0);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t t = words[q] ^ 0x80808080u;
            const uint32_t w01 = hsub2_bits(__byte_perm(t, 0x64646464u, 0x4140u), 0x64806480u);  // channels 4q, 4q+1
            const uint32_t w23 = hsub2_bits(__byte_perm(t, 0x64646464u, 0x4342u), 0x64806480u);  // 4q+2, 4q+3
#pragma unroll
            for (int m = 0; m < kM; ++m) {
              acc[m][4 * q + 0] = fma_h_lo(xv[m], w01, acc[m][4 * q + 0]);
              acc[m][4 * q + 1] = fma_h_hi(xv[m], w01, acc[m][4 * q + 1]);
              acc[m][4 * q + 2] = fma_h_lo(xv[m], w23, acc[m][4 * q + 2]);
              acc[m][4 * q + 3] = fma_h_hi(xv[m], w23, acc[m][4 * q + 3]);
            }
          }
        } else {
          // stored row r holds k = 2r (low nibbles) and k = 2r + 1 (high nibbles)
          uint16_t x0[kM], x1[kM];
#pragma unroll
          for (int m = 0; m < kM; ++m) {
            x0[m] = row_ok ? xs[m * kspan + kl] : uint16_t(0);
            x1[m] = row_ok ? xs[m * kspan + kl + 1] : uint16_t(0);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            // byte j = channel 4q + j; masks pick channels (4q, 4q+2), then
            // (4q+1, 4q+3) after an 8-bit shift.
            const uint32_t t = words[q] ^ 0x88888888u;  // every nibble q -> q + 8
            const uint32_t u = t >> 8;
            const uint32_t lo02 = hsub2_bits((t & 0x000F000Fu) | 0x64006400u, 0x64086408u);
            const uint32_t lo13 = hsub2_bits((u & 0x000F000Fu) | 0x64006400u, 0x64086408u);
            const uint32_t hi02 = hfma2_bits((t & 0x00F000F0u) | 0x64006400u, 0x2C002C00u, 0xD480D480u);
            const uint32_t hi13 = hfma2_bits((u & 0x00F000F0u) | 0x64006400u, 0x2C002C00u, 0xD480D480u);
#pragma unroll
            for (int m = 0; m < kM; ++m) {
              acc[m][4 * q + 0] = fma_h_lo(x1[m], hi02, fma_h_lo(x0[m], lo02, acc[m][4 * q + 0]));
              acc[m][4 * q + 1] = fma_h_lo(x1[m], hi13, fma_h_lo(x0[m], lo13, acc[m][4 * q + 1]));
              acc[m][4 * q + 2] = fma_h_hi(x1[m], hi02, fma_h_hi(x0[m], lo02, acc[m][4 * q + 2]));
              acc[m][4 * q + 3] = fma_h_hi(x1[m], hi13, fma_h_hi(x0[m], lo13, acc[m][4 * q + 3]));
            }
          }
        }
      }
      if (kQ == kInt4G128 && ((r + U) % 64 == 0 || r + U >= wr1)) {
        // A 128-wide group (64 stored rows) ends here: scale its sums.
        const __half* sg = a.scale + static_cast<int64_t>(r / 64) * a.lds + n0;
        const uint4 s0 = *reinterpret_cast<const uint4*>(sg);
        const uint4 s1 = *reinterpret_cast<const uint4*>(sg + 8);
        const __half* sh0 = reinterpret_cast<const __half*>(&s0);
        const __half* sh1 = reinterpret_cast<const __half*>(&s1);
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
          const float sc = __half2float(i < 8 ? sh0[i] : sh1[i - 8]);
#pragma unroll
          for (int m = 0; m < kM; ++m) {
            tot[m][i] = fmaf(acc[m][i], sc, tot[m][i]);
            acc[m][i] = 0.f;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) cur[u] = nxt[u];
    }
  }
  if (kQ == kInt4G128) {
#pragma unroll
    for (int m = 0; m < kM; ++m)
#pragma unroll
      for (int i = 0; i < CPL; ++i) acc[m][i] = tot[m][i];
  }
  __syncthreads();  // X slice no longer needed: the reduction reuses the buffer

  // CTA reduction over the warps, one output row m at a time; the slice's
  // sums go to Y (single slice) or to partial[sl].
  const bool single = slices == 1;
  for (int m = 0; m < a.M && m < kM; ++m) {
#pragma unroll
    for (int i = 0; i < CPL; ++i) gsm[warp * kGvWarpStride + lane * 17 + i] = acc[m][i];
    __syncthreads();
    for (int c = threadIdx.x; c < kGvChannels; c += Cfg::kThreads) {
      const int n = cb * kGvChannels + c;
      if (n < a.N) {
        const int off = (c / CPL) * 17 + (c % CPL);
        float s = 0.f;
#pragma unroll 8
        for (int w = 0; w < NW; ++w) s += gsm[w * kGvWarpStride + off];
        if (single) {
          if (kQ == kInt8 && a.scale != nullptr) {
            s *= __half2float(a.scale[n]);
          } else if (kQ == kInt8 && a.tscale != nullptr) {
            s *= __ldg(a.tscale);
          }
          a.Y[static_cast<int64_t>(m) * a.ldy + n] = s;
        } else {
          a.partial[(static_cast<int64_t>(sl) * a.M + m) * a.N + n] = s;
        }
      }
    }
    __syncthreads();
  }
  if (single) return;

  // The last CTA of this channel block adds the slices in order. The CTA's
  // partial stores are ordered before the ticket by the barrier and the
  // ticket's release; its acquire orders the last CTA's loads after every
  // other CTA's release.
  __syncthreads();
  if (threadIdx.x == 0) {
    int prev;
    asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(prev) : "l"(a.counters + cb) : "memory");
    is_last = prev == slices - 1;
  }
  __syncthreads();
  if (!is_last) return;
  for (int o = threadIdx.x; o < a.M * kGvChannels; o += Cfg::kThreads) {
    const int m = o / kGvChannels;
    const int n = cb * kGvChannels + (o % kGvChannels);
    if (n >= a.N) continue;
    // Sixteen slices' loads in flight at a time, summed in slice order.
    const float* src = a.partial + static_cast<int64_t>(m) * a.N + n;
    const int64_t step = static_cast<int64_t>(a.M) * a.N;
    float s = 0.f;
    for (int k = 0; k < slices; k += 16) {
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = (k + i < slices) ? __ldcg(src + (k + i) * step) : 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) s += v[i];
    }
    if (kQ == kInt8 && a.scale != nullptr) {
      s *= __half2float(a.scale[n]);
    } else if (kQ == kInt8 && a.tscale != nullptr) {
      s *= __ldg(a.tscale);
    }
    a.Y[static_cast<int64_t>(m) * a.ldy + n] = s;
  }
  if (threadIdx.x == 0) a.counters[cb] = 0;  // ready for the next launch on this stream
}

// Work split of the small-M path: channel blocks, stored rows per K slice and
// slices. One wave of one CTA per SM: the K slices per channel block fill the
// SMs, and few slices keep the final in-order sum short. `fits`: the slice of
// X staged in the reduction buffer fits in shared memory.
struct GvPlan {
  int nblk, rows_per_slice, slices;
  bool fits;
};
template <int kQ, int kM>
GvPlan gemv_plan(const QProblem& p) {
  using Cfg = GvCfg<kQ, kM>;
  GvPlan g{};
  const int rows = kQ == kInt8 ? p.K : p.K / 2;
  g.nblk = (p.N + kGvChannels - 1) / kGvChannels;
  const int want = std::max(1, Cfg::kCtasPerSm * sm_count() / g.nblk);
  const int unit = 4 * Cfg::kWarps;  // rows per slice: a whole number of 4-row batches per warp
  int rps = (rows + want - 1) / want;
  rps = (rps + unit - 1) / unit * unit;
  g.rows_per_slice = rps;
  g.slices = (rows + rps - 1) / rps;
  g.fits = static_cast<int64_t>(kM) * (kQ == kInt8 ? 1 : 2) * rps * 4 <= Cfg::kSmemBytes && g.slices <= 65535;
  return g;
}

template <int kQ, int kM>
int launch_gemv(const QProblem& p, cudaStream_t stream) {
  using Cfg = GvCfg<kQ, kM>;
  GvArgs a{};
  a.X = static_cast<const __half*>(p.X);
  a.ldx = p.ldx;
  a.W = static_cast<const uint8_t*>(p.W);
  a.ldw = p.ldw;
  a.scale = static_cast<const __half*>(p.scale);
  a.lds = p.lds;
  a.tscale = kQ == kInt8 ? p.tscale : nullptr;
  a.Y = p.Y;
  a.ldy = p.ldy;
  a.M = p.M;
  a.N = p.N;
  a.rows = kQ == kInt8 ? p.K : p.K / 2;
  auto kern = wq_gemv_kernel<kQ, kM>;
  int rc = kernel_setup(reinterpret_cast<const void*>(kern), Cfg::kSmemBytes, nullptr);
  if (rc != NESO_OK) return rc;
  const GvPlan g = gemv_plan<kQ, kM>(p);
  if (!g.fits) return fail(NESO_ERR_UNSUPPORTED, "K slice too long for the small-M path");
  const int nblk = g.nblk, slices = g.slices;
  a.rows_per_slice = g.rows_per_slice;
  if (slices > 1) {
    void* ws = nullptr;
    rc = stream_workspace(stream, static_cast<size_t>(slices) * p.M * p.N * sizeof(float), &ws);
    if (rc != NESO_OK) return rc;
    a.partial = static_cast<float*>(ws);
    int* ctr = nullptr;
    rc = stream_counters(stream, &ctr);
    if (rc != NESO_OK) return rc;
    a.counters = ctr + kGemvCounterBase;
  }
  cudaError_t e = launch_pdl(kern, dim3(nblk, slices, 1), dim3(Cfg::kThreads), Cfg::kSmemBytes, stream, a);
  if (e != cudaSuccess) return cuda_fail(e, "small-M GEMV launch");
  return ok();
}

// The small-M path applies when M is small, rows are 16-byte aligned and the
// channel blocks fit the per-stream counter slots.
bool gemv_eligible(const QProblem& p) {
  const int max_m = p.kind == kInt8 ? 4 : 2;
  const int nblk = (p.N + kGvChannels - 1) / kGvChannels;
  // int4 reads each lane's 16 group scales with two 16-byte loads.
  const bool scales_ok = p.kind == kInt8 || (reinterpret_cast<uintptr_t>(p.scale) & 15u) == 0;
  if (!(p.M <= max_m && p.N % 16 == 0 && p.ldw % 16 == 0 && (reinterpret_cast<uintptr_t>(p.W) & 15u) == 0 &&
        scales_ok && nblk <= kGemvCounterEnd - kGemvCounterBase)) {
    return false;
  }
  // Long K: a slice of X must fit in shared memory, else the tensor-core path runs.
  if (p.kind == kInt8) {
    return p.M == 1 ? gemv_plan<kInt8, 1>(p).fits : p.M == 2 ? gemv_plan<kInt8, 2>(p).fits : gemv_plan<kInt8, 4>(p).fits;
  }
  return p.M == 1 ? gemv_plan<kInt4G128, 1>(p).fits : gemv_plan<kInt4G128, 2>(p).fits;
}

int run_gemv(const QProblem& p, cudaStream_t stream) {
  if (p.kind == kInt8) {
    if (p.M == 1) return launch_gemv<kInt8, 1>(p, stream);
    if (p.M == 2) return launch_gemv<kInt8, 2>(p, stream);
    return launch_gemv<kInt8, 4>(p, stream);
  }
  if (p.M == 1) return launch_gemv<kInt4G128, 1>(p, stream);
  return launch_gemv<kInt4G128, 2>(p, stream);
}

template <int kQ>
int dispatch_wq(const QProblem& p, cudaStream_t stream) {
  if (p.M <= 16) return p.pair ? launch_wq<kQ, true, 16, 2>(p, stream) : launch_wq<kQ, true, 16>(p, stream);
  if (p.M <= 32) return launch_wq<kQ, true, 32>(p, stream);
  if (p.M <= 64) return launch_wq<kQ, true, 64>(p, stream);
  if constexpr (kQ == kInt4G128) {
    if (p.M <= 128) return launch_wq<kQ, true, 128>(p, stream);
  }
  if (p.rows2) {
    // 256-row units: W8A16 with paired channel tiles (256 x 256), W4A16 with
    // one tile (256 x 128; its fp16 w_hi and E5M2 w_lo tiles and E5M2 X
    // blocks leave no room for pairs).
    if constexpr (kQ == kInt8) {
      return launch_wq<kQ, false, 256, 2>(p, stream);
    } else {
      return launch_wq<kQ, false, 256, 1>(p, stream);
    }
  }
  if (p.pair) return launch_wq<kQ, false, 128, 2>(p, stream);
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
  } else {
    if (p.K % 128 != 0) return fail(NESO_ERR_UNSUPPORTED, "int4 group-128 needs K %% 128 == 0 (K=%d)", p.K);
    if (p.scale == nullptr) return fail(NESO_ERR_INVALID_ARG, "null scales");
    if (p.lds < p.N || (p.lds * 2) % 16 != 0) {
      return fail(NESO_ERR_MISALIGNED, "scale row stride must be >= N, multiple of 8");
    }
  }
  if (gemv_eligible(p)) return run_gemv(p, stream);
  QProblem q = p;
  int rc = device_status(&q.st);
  if (rc != NESO_OK) return rc;
  plan_splits(q, sm_count());
  if (q.splits > 1) {
    void* ws = nullptr;
    rc = stream_workspace(stream, static_cast<size_t>(q.splits) * q.M * q.N * sizeof(float), &ws);
    if (rc != NESO_OK) return rc;
    q.partial = static_cast<float*>(ws);
  }
  return q.kind == kInt8 ? dispatch_wq<kInt8>(q, stream) : dispatch_wq<kInt4G128>(q, stream);
}

// ------------------------------------ per-tensor scale, int32-held weights --
// tests/test_advanced12.py:19-48 w8a16_matmul_kernel: C = (A . f16(B)) * scale[0]
// with one fp32 scale; the reference's test holds the int8 values in an int32
// tensor (:186). Those are narrowed to int8 rows of `ldo` bytes first (values
// outside [-128, 127] saturate; the kernel's contract is int8 data).
__global__ void narrow_i32_to_i8_kernel(const int32_t* __restrict__ b, int64_t ldb, int K, int N,
                                        int8_t* __restrict__ out, int64_t ldo) {
  const int64_t quads = static_cast<int64_t>(K) * (N / 4);
  const bool vec = (ldb % 4 == 0) && ((reinterpret_cast<uintptr_t>(b) & 15u) == 0);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < quads;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t k = i / (N / 4);
    const int n = static_cast<int>(i % (N / 4)) * 4;
    int v[4];
    if (vec) {
      const int4 q = __ldg(reinterpret_cast<const int4*>(b + k * ldb + n));
      v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = __ldg(b + k * ldb + n + j);
    }
    uint32_t packed = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) packed |= (static_cast<uint32_t>(max(-128, min(127, v[j]))) & 0xFFu) << (8 * j);
    *reinterpret_cast<uint32_t*>(out + k * ldo + n) = packed;
  }
}

// Reference-grid and stride checks shared by both storage forms of
// w8a16_matmul_kernel (the grid is (cdiv(M, BLOCK_M), cdiv(N, BLOCK_N)), as
// for matmul_kernel).
int check_w8a16_tensor_scale(int M, int N, int K, int stride_ak, int stride_bn, int stride_cn, int BLOCK_M,
                             int BLOCK_N, int BLOCK_K, uint32_t gx, uint32_t gy, uint32_t gz, const float* scale) {
  if (BLOCK_M <= 0 || BLOCK_N <= 0 || BLOCK_K <= 0) return fail(NESO_ERR_INVALID_ARG, "BLOCK_* must be positive");
  if (M < 0 || N < 0 || K < 0) return fail(NESO_ERR_INVALID_ARG, "negative size");
  const uint32_t gm = static_cast<uint32_t>((static_cast<int64_t>(M) + BLOCK_M - 1) / BLOCK_M);
  const uint32_t gn = static_cast<uint32_t>((static_cast<int64_t>(N) + BLOCK_N - 1) / BLOCK_N);
  if (gx != gm || gy != gn || gz != 1) {
    return fail(NESO_ERR_GRID, "grid (%u,%u,%u) != (cdiv(M,BLOCK_M)=%u, cdiv(N,BLOCK_N)=%u, 1)", gx, gy, gz, gm,
                gn);
  }
  if (stride_ak != 1 || stride_bn != 1 || stride_cn != 1) {
    return fail(NESO_ERR_UNSUPPORTED, "only unit inner strides are supported (stride_ak=%d stride_bn=%d "
                                      "stride_cn=%d)", stride_ak, stride_bn, stride_cn);
  }
  if (scale == nullptr && M > 0 && N > 0) return fail(NESO_ERR_INVALID_ARG, "null scale_ptr");
  return NESO_OK;
}

// ---------------------------------------------------- allocation-free entry --
// Scratch for neso_w8a16_matmul_mnk_noalloc: the split-K partial sums and a
// status block, in fixed device arrays that exist in every GPU's copy of this
// library from load until process exit. Host code never dereferences these
// names (on the host they are only stand-ins for the device symbols); their
// device addresses come from cudaGetSymbolAddress, once per device.
constexpr size_t kNoAllocScratchFloats = size_t(1) << 20;  // 4 MiB of fp32 partial sums
static __device__ __align__(256) float g_noalloc_partial[kNoAllocScratchFloats];
static __device__ __align__(256) int g_noalloc_status[16];

struct NoAllocDevice {
  std::once_flag once;
  float* partial = nullptr;
  int* status = nullptr;
  cudaError_t err = cudaSuccess;
};
NoAllocDevice g_noalloc_dev[64];

// Device addresses of the fixed scratch for the current device (first call
// per device resolves them; it must run before any stream capture).
int noalloc_scratch(float** partial, int** status) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(NESO_ERR_NO_DEVICE, "device ordinal %d out of range", dev);
  NoAllocDevice& d = g_noalloc_dev[dev];
  std::call_once(d.once, [&d]() {
    void* p = nullptr;
    void* q = nullptr;
    d.err = cudaGetSymbolAddress(&p, g_noalloc_partial);
    if (d.err == cudaSuccess) d.err = cudaGetSymbolAddress(&q, g_noalloc_status);
    if (d.err == cudaSuccess) {
      d.partial = static_cast<float*>(p);
      d.status = static_cast<int*>(q);
    }
  });
  if (d.err != cudaSuccess) return cuda_fail(d.err, "cudaGetSymbolAddress(no-allocation scratch)");
  *partial = d.partial;
  *status = d.status;
  return NESO_OK;
}

}  // namespace

// Status block of the allocation-free entry point on the current device
// (4 ints: code, where, block, thread); read without allocating.
int noalloc_status_read(int* host4) {
  float* partial = nullptr;
  int* status = nullptr;
  int rc = noalloc_scratch(&partial, &status);
  if (rc != NESO_OK) return rc;
  cudaError_t e = cudaMemcpy(host4, status, 4 * sizeof(int), cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? NESO_OK : cuda_fail(e, "reading the no-allocation status block");
}

// Zeroes that status block on the current device (neso_clear_device_status).
int noalloc_status_clear() {
  float* partial = nullptr;
  int* status = nullptr;
  int rc = noalloc_scratch(&partial, &status);
  if (rc != NESO_OK) return rc;
  cudaError_t e = cudaMemset(status, 0, 16 * sizeof(int));
  return e == cudaSuccess ? NESO_OK : cuda_fail(e, "clearing the no-allocation status block");
}

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


int neso_w8a16_matmul_kernel(const void* a_ptr, const int8_t* b_int8_ptr, float* c_ptr, const float* scale_ptr,
                             int32_t M, int32_t N, int32_t K, int32_t stride_am, int32_t stride_ak, int32_t stride_bk,
                             int32_t stride_bn, int32_t stride_cm, int32_t stride_cn, int32_t BLOCK_M, int32_t BLOCK_N,
                             int32_t BLOCK_K, uint32_t grid_x, uint32_t grid_y, uint32_t grid_z,
                             neso_stream_t stream) {
  int rc = check_w8a16_tensor_scale(M, N, K, stride_ak, stride_bn, stride_cn, BLOCK_M, BLOCK_N, BLOCK_K, grid_x,
                                    grid_y, grid_z, scale_ptr);
  if (rc != NESO_OK) return rc;
  QProblem p{};
  p.X = a_ptr; p.ldx = stride_am;
  p.W = b_int8_ptr; p.ldw = stride_bk;
  p.scale = nullptr; p.lds = 0;
  p.tscale = scale_ptr;
  p.Y = c_ptr; p.ldy = stride_cm;
  p.M = M; p.N = N; p.K = K;
  p.kind = kInt8;
  return run_wq(p, as_stream(stream));
}

int neso_w8a16_matmul_kernel_i32(const void* a_ptr, const int32_t* b_int8_ptr, float* c_ptr, const float* scale_ptr,
                                 int32_t M, int32_t N, int32_t K, int32_t stride_am, int32_t stride_ak,
                                 int32_t stride_bk, int32_t stride_bn, int32_t stride_cm, int32_t stride_cn,
                                 int32_t BLOCK_M, int32_t BLOCK_N, int32_t BLOCK_K, uint32_t grid_x, uint32_t grid_y,
                                 uint32_t grid_z, neso_stream_t stream) {
  int rc = check_w8a16_tensor_scale(M, N, K, stride_ak, stride_bn, stride_cn, BLOCK_M, BLOCK_N, BLOCK_K, grid_x,
                                    grid_y, grid_z, scale_ptr);
  if (rc != NESO_OK) return rc;
  if (M == 0 || N == 0) return ok();
  if (stride_bk < N) return fail(NESO_ERR_INVALID_ARG, "stride_bk %d < N %d", stride_bk, N);
  if (N % 16 != 0) return fail(NESO_ERR_UNSUPPORTED, "int32-held weights need N %% 16 == 0 (N=%d)", N);
  cudaStream_t st = as_stream(stream);
  const int64_t ldw = N;  // int8 rows on 16-byte boundaries for TMA
  int8_t* w8 = nullptr;
  if (K > 0) {
    if (b_int8_ptr == nullptr) return fail(NESO_ERR_INVALID_ARG, "null input");
    void* ws = nullptr;
    rc = stream_workspace(st, static_cast<size_t>(K) * ldw, &ws, kWorkspaceInputs);
    if (rc != NESO_OK) return rc;
    w8 = static_cast<int8_t*>(ws);
    const int64_t quads = static_cast<int64_t>(K) * (N / 4);
    const int blocks = static_cast<int>(std::min<int64_t>((quads + 255) / 256, 8 * sm_count()));
    narrow_i32_to_i8_kernel<<<blocks, 256, 0, st>>>(b_int8_ptr, stride_bk, K, N, w8, ldw);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "int32 -> int8 weight launch");
  }
  QProblem p{};
  p.X = a_ptr; p.ldx = stride_am;
  p.W = w8; p.ldw = ldw;
  p.scale = nullptr; p.lds = 0;
  p.tscale = scale_ptr;
  p.Y = c_ptr; p.ldy = stride_cm;
  p.M = M; p.N = N; p.K = K;
  p.kind = kInt8;
  return run_wq(p, st);
}

int neso_w8a16_matmul_mnk_noalloc(const void* X, const int8_t* W, const void* scale, float* Y, int32_t M, int32_t N,
                                  int32_t K, neso_stream_t stream) {
  // Same problem and result as neso_w8a16_matmul_mnk, for callers that must
  // not allocate device memory: the split-K scratch is the fixed array above
  // and no CUDA allocation is made (the first call on a device resolves the
  // array's address, see noalloc_scratch).
  if (M < 0 || N < 0 || K < 0) return fail(NESO_ERR_INVALID_ARG, "negative size");
  if (M == 0 || N == 0) return ok();
  if (Y == nullptr) return fail(NESO_ERR_INVALID_ARG, "null output");
  if (K == 0) {  // an empty sum: Y = 0, as the allocating entry point writes it
    zero_y_kernel<<<256, 256, 0, as_stream(stream)>>>(Y, N, M, N);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : cuda_fail(e, "zero launch");
  }
  if (X == nullptr || W == nullptr) return fail(NESO_ERR_INVALID_ARG, "null input");
  if (K % 8 != 0 || N % 16 != 0) {
    return fail(NESO_ERR_MISALIGNED, "noalloc W8A16 needs K %% 8 == 0 and N %% 16 == 0 (K=%d N=%d)", K, N);
  }
  QProblem q{};
  q.X = X; q.ldx = K;
  q.W = W; q.ldw = N;
  q.scale = scale; q.lds = 0;
  q.Y = Y; q.ldy = N;
  q.M = M; q.N = N; q.K = K;
  q.kind = kInt8;
  // The planner only considers K splits whose partial sums fit the fixed
  // scratch, falling back to fewer splits (one split needs none).
  plan_splits(q, sm_count(), kNoAllocScratchFloats);
  const size_t need = q.splits > 1 ? static_cast<size_t>(q.splits) * M * N : 0;
  if (need > kNoAllocScratchFloats) {  // guard: the planner above never returns such a plan
    return fail(NESO_ERR_UNSUPPORTED,
                "noalloc W8A16: M=%d N=%d needs %zu split-K partial floats (%d splits), above the fixed scratch "
                "of %zu floats; use neso_w8a16_matmul_mnk", M, N, need, q.splits, kNoAllocScratchFloats);
  }
  float* partial = nullptr;
  int* status = nullptr;
  int rc = noalloc_scratch(&partial, &status);
  if (rc != NESO_OK) return rc;
  // The partial sums need no clearing: every split writes all of its M x N
  // entries. The status block records the first timed-out wait since the last
  // neso_clear_device_status, like the main status word.
  q.st.word = status;
  q.st.budget_ns = kWaitBudgetNs;
  q.partial = need > 0 ? partial : nullptr;
  return dispatch_wq<kInt8>(q, as_stream(stream));
}

}  // extern "C"
