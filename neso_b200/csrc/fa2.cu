// Flash Attention 2 forward on sm_100a (tcgen05 + TMA + TMEM).
//
// Reference kernels:
//   tests/test_flash_attention.py:79-247  flash_attention_fwd(Q,K,V,O,N,stride_qo,
//       stride_kv,scale): single head, fp16 Q/K/V, fp32 O; online softmax per
//       BN-key block; P rounded to the input dtype before P.V (:139-142);
//       O = O / l at the end.
//   tests/test_rel_pos_fa2.py:155-252  rel_pos_fa2_fwd: head on grid y, dense
//       fp16 bias added before the scale, scores = (QK + bias) * scale (:202-206),
//       fp16 O.
//   Extensions with no reference kernel: [B,H,S,D] multi-head, causal masking,
//       and an fp32 relative-position table [H, 2S-1] indexed i - j + S - 1.
//
// Work unit: one (batch*head, 256 query rows) = two 128-row Q tiles that
// ping-pong so the tensor core runs one tile's MMAs while the other tile's
// softmax runs on the CUDA cores. Keys are consumed in 128-key blocks. Two
// kernels share this design and the host picks the faster one per head dim
// (measured on B200):
//   D = 64   fa2_pair_kernel: one 128-row tile at a time per CTA and two
//            CTAs per SM (256 TMEM columns, 100 KB of shared memory each):
//            the tiles of the two CTAs overlap as the ping-pong pair does.
//            Non-causal, each CTA walks the (head, query tile) units
//            blockIdx.x, blockIdx.x + gridDim.x, ... (persistent: the next
//            tile's Q load and first QK run under this tile's last blocks
//            and epilogue); causal, it processes tiles qb and nq-1-qb.
//   D = 128  fa2_persistent_kernel: one two-tile CTA per SM walks units
//            handed out from a per-launch counter.
// The description below is of the two-tile form; the one-tile form drops
// warps 8-11 and the turn handshake.
//   warp 0       TMA producer: Q tiles once, then K_j / V_j into KV rings.
//   warp 1       single-thread tcgen05.mma issuer of S_t = Q_t . K_j^T (SS,
//                M=128 N=128 K=16 steps, fp32 in TMEM); in the D = 128 kernel
//                also of O_t += P_t . V_j, each PV_t(j) followed at once by
//                S_t(j+1)
//   warp 3       one-tile kernel: single-thread tcgen05.mma issuer of
//                O += P . V_j (TS: P from TMEM, V MN-major from smem)
//   warp 2       TMEM allocator (512 columns).
//   warps 4-7    softmax + epilogue for tile 0; warps 8-11 for tile 1. Thread
//                r owns query row r: it reads its S row from TMEM, computes the
//                row max / exp2 / row sum in registers, writes fp16 P back to
//                TMEM and, only when the running max grew by more than 2^8,
//                rescales its O row in TMEM (lazy rescaling: exact in real
//                arithmetic because O and l always share one reference max).
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D);
//   D = 64: P0/P1 in [384,448)/[448,512); D = 128: P_t aliases the first 64
//   columns of S_t, and QK_t(j+1) is issued after PV_t(j) by the same thread
//   (tcgen05.mma operations of one thread run in issue order).
//   One-tile form (D = 64): S [0,128) O [128,192) P [192,256).
// Relative-position table: the 32 rows of a softmax warp need 159
// consecutive table entries per 128-key block; the warp stages them in its
// own shared-memory window (global loads issued one block ahead) and each row
// reads its 128 values from there, adding them two keys per packed FMA
// (measured S=2048, B=H=16 against 128 scattered global loads per row and
// block: D=64 152 -> 506 TFLOP/s, D=128 614 -> 720-740; causal 113 -> 399 and
// 422 -> 514-593).
#include <algorithm>
#include <cmath>

#include "runtime.h"

namespace neso {
namespace {

// Register split: warpgroup 0 (TMA, MMA, TMEM warps) shrinks to
// FaCfg::regs_low(), the softmax warpgroups grow to kRegsHigh; the host checks
// that the split fits the block's launch pool.
constexpr uint32_t kRegsHigh = 216;
// The persistent kernel's producer and MMA issuer keep per-unit state across
// units and get more registers; 128 * 88 + 256 * 208 fills the launch pool
// (168 registers x 384 threads).
constexpr uint32_t kRegsLowPersistent = 88;
constexpr uint32_t kRegsHighPersistent = 208;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale only when max grows by > 2^8
constexpr int kUnitRing = 4;      // unit indices the persistent producer may publish ahead
constexpr int kUnitReaders = 9;  // the MMA issuer and the 8 softmax warps

enum BiasMode : int { kBiasNone = 0, kBiasTable = 1, kBiasDense = 2 };

// z + (low or high fp16 half of b2), the half widened exactly: one mixed-
// precision add instead of a conversion and an fp32 add.
__device__ __forceinline__ float add_f16_lo(uint32_t b2, float z) {
  float d;
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %1;\n\tadd.rn.f32.f16 %0, l, %2;\n\t}" : "=f"(d) : "r"(b2), "f"(z));
  return d;
}
__device__ __forceinline__ float add_f16_hi(uint32_t b2, float z) {
  float d;
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %1;\n\tadd.rn.f32.f16 %0, h, %2;\n\t}" : "=f"(d) : "r"(b2), "f"(z));
  return d;
}

// Relative-position table of one 128-row x 128-key block: row i, key c use
// table[h, d0 + i - c + 127] with d0 = (tile row 0) - (key 0) - 127 + S - 1.
// The 32 rows of softmax warp q need the 159 consecutive entries from
// d0 + 32 q: the warp stages them, scaled by log2(e), in its own 160-float
// window (lane l row: window[l + 127 - c], consecutive lanes on consecutive
// banks), from registers loaded one block ahead so the L2 latency hides
// under the current block. Nothing is shared between warps. Entries outside
// [0, 2S - 1) only meet rows or keys past S and are 0.
__device__ __forceinline__ void table_window_load(float (&v)[5], const float* ttab, int d0, int ncols, int lane) {
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    const int u = lane + 32 * i;
    const int col = d0 + u;
    v[i] = (u < 159 && col >= 0 && col < ncols) ? __ldg(ttab + col) : 0.f;
  }
}
// Stores the window and returns this lane's row pointer (read at [-c]).
__device__ __forceinline__ const float* table_window_store(float* win, const float (&v)[5], int lane) {
  __syncwarp();  // every lane has read the previous block's window
#pragma unroll
  for (int i = 0; i < 5; ++i) win[lane + 32 * i] = v[i] * kLog2e;
  __syncwarp();
  return win + lane + 127;
}

// kT = Q tiles per CTA: 2 (ping-pong pair, one CTA per SM) or 1 (two CTAs
// per SM, each with half the TMEM and shared memory).
template <int D, int kT = 2>
struct FaCfg {
  static constexpr int kThreads = 128 * (1 + kT);
  __host__ __device__ static constexpr int min_blocks() { return kT == 1 ? 2 : 1; }
  static constexpr int kChunks = D / 64;           // 128-byte TMA boxes per row
  static constexpr int kTileBytes = 128 * D * 2;   // one Q, K or V tile
  static constexpr int kStages = (D == 64 && kT == 2) ? 3 : 2;
  static constexpr int kQBuffers = 1;  // persistent kernel: Q tiles per unit in flight
  static constexpr bool kAliasP = (D > 64);
  // Warpgroup 0 register budget; 128 * kRegsLow + 128 * kT * kRegsHigh must
  // fit the launch pool (kThreads x registers per thread).
  __host__ __device__ static constexpr uint32_t regs_low() { return kT == 1 ? 40 : 56; }
  __host__ __device__ static constexpr uint32_t s_col(int t) { return t ? 128u : 0u; }
  __host__ __device__ static constexpr uint32_t o_col(int t) {
    return kT == 1 ? 128u : (t ? 256u + D : 256u);
  }
  __host__ __device__ static constexpr uint32_t p_col(int t) {
    return kAliasP ? s_col(t) : (kT == 1 ? 128u + D : (t ? 256u + 2 * D + 64 : 256u + 2 * D));
  }
  static constexpr uint32_t kPHalfStride = 32u;  // P columns are contiguous (64 per tile)
  static constexpr int kTmemCols = kT == 1 ? 256 : 512;
  // Persistent kernel: O staging for TMA stores, 32 rows x 128 bytes per
  // softmax warp (the K/V ring is busy with the next unit meanwhile).
  static constexpr int kOutBytes = kT == 2 ? 4 * kT * 4096 : 0;
  // One-tile kernels: relative-position table windows, 160 floats per
  // softmax warp (the persistent kernel uses its O staging blocks).
  static constexpr int kTableBytes = kT == 1 ? 4 * 160 * 4 : 0;
  static constexpr int kSmemBytes =
      (kT * kQBuffers + 2 * kStages) * kTileBytes + kOutBytes + kTableBytes + 1024 + 512;
};

// Dynamic shared memory of the one-tile kernel: Q, the K/V ring, one block
// per softmax warp, the table windows and the barriers. The softmax warp's
// block is its 4 KB O staging, or with a dense bias 8 KB that hold its 32 rows
// of the next key block's bias (two 64-key TMA boxes) and, in its first 4 KB,
// the O staging. Two such CTAs fill an SM's 228 KB only without the 1 KB of
// alignment slack, so the dense-bias kernel checks its base instead.
template <int D, int kBias>
constexpr int pair_smem_bytes() {
  using Cfg = FaCfg<D, 1>;
  return kBias == kBiasDense ? (1 + 2 * Cfg::kStages) * Cfg::kTileBytes + 4 * 8192 + 512
                             : Cfg::kSmemBytes + 4 * 4096;
}

struct FaArgs {
  void* O;
  int64_t o_row;   // elements
  int64_t o_head;  // elements
  int S;
  int H;
  float qk_log2;  // scale * log2(e)
  const float* table;       // kBiasTable: [H, 2S-1] fp32
  const __half* bias;       // kBiasDense: [BH][S][S] fp16 (row stride bias_row)
  int64_t bias_head, bias_row;
  int num_qblocks;
  int BH;
  int out_f16;
  // Persistent kernel: [0] next unit ticket, [1] CTAs finished. Zero at
  // launch; the last CTA to finish puts both back to zero for the next launch
  // on the stream.
  int* unit_counter;
  DevStatus st;
};

// Query tiles one after the other in one CTA (the roles above, one tile's
// TMEM layout). Causal: tiles bx and nq-1-bx of one head, so every
// CTA has nq+1 key blocks (S=2048 494 -> 515 TFLOP/s, S=512 214 -> 231
// against one tile per CTA). Non-causal: a persistent walk over the (head,
// query tile) units, two CTAs per SM (B=H=16 D=64: S=512 364 -> 431,
// S=1024 535 -> 559, S=2048 639 -> 647 against one tile per CTA). The CTA's
// prologue and launch are paid once, the next tile's first QK runs while
// this tile's epilogue drains O, and O leaves through a dedicated staging
// area (the K/V ring is busy with the next tile by then). Every mbarrier
// phase runs over the CTA's blocks of all its tiles (running block index
// g); q_empty hands the single Q buffer to the next tile's load after the
// last QK, o_free the O columns to the next tile's first PV after the
// epilogue has read them.
template <int D, bool kCausal, int kBias>
__global__ void __launch_bounds__(FaCfg<D, 1>::kThreads, 2)
    fa2_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                    const __grid_constant__ CUtensorMap tmB, FaArgs a) {
  using Cfg = FaCfg<D, 1>;
  constexpr int kT = 1;
  constexpr int KS = Cfg::kStages;
  constexpr bool kBiasTma = kBias == kBiasDense;
  constexpr int kWarpBytes = kBiasTma ? 8192 : 4096;  // per softmax warp, see pair_smem_bytes
  extern __shared__ uint8_t smem_raw[];
  if constexpr (kBiasTma) {
    // No alignment slack in this layout (see pair_smem_bytes).
    if ((smem_u32(smem_raw) & 1023u) != 0) {
      if (threadIdx.x == 0) record_error(a.st, kDevSmemMisaligned, 0x13f0);
      return;
    }
  }
  uint8_t* smem = kBiasTma ? smem_raw
                           : reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                        ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Cfg::kTileBytes;                // KS tiles
  uint8_t* sV = sK + KS * Cfg::kTileBytes;           // KS tiles
  uint8_t* sOut = sV + KS * Cfg::kTileBytes;         // kWarpBytes per softmax warp
  float* tb_base = reinterpret_cast<float*>(sOut + 4 * kWarpBytes);  // table windows
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + 4 * kWarpBytes + (kBiasTma ? 0 : Cfg::kTableBytes));
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;
  uint64_t* k_empty = k_full + KS;
  uint64_t* v_full = k_empty + KS;
  uint64_t* v_empty = v_full + KS;
  uint64_t* s_full = v_empty + KS;   // [1]
  uint64_t* p_full = s_full + 1;     // [1]
  uint64_t* o_done = p_full + 1;     // [1]
  uint64_t* s_free = o_done + 1;     // [1] softmax has read S (4 warps)
  uint64_t* o_free = s_free + 1;     // [1] epilogue has read O (4 warps)
  uint64_t* mma_done = o_free + 1;   // [2] one per MMA issuer
  uint64_t* turn = mma_done + 2;     // [4] dense bias of softmax warp q arrived (no exp turns here)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(turn + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* never_flag = abort_flag + 1;  // stays 0: drain waits ignore the abort

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int S = a.S;
  const int nq = a.num_qblocks;
  const int bx = static_cast<int>(blockIdx.x);
  const int nkv = (S + 127) / 128;
  // Work list. Causal: query tiles nq-1-bx (the heavier, first) and bx of head
  // blockIdx.y, so every CTA has nq + 1 key blocks. Otherwise a persistent
  // walk over the (head, query tile) units bx, bx + gridDim.x, ...: the CTA
  // pays its prologue once, the next tile's Q load and first QK run under
  // this tile's last blocks and epilogue, and the CTAs running at one time
  // hold consecutive units, so they share K/V in L2.
  const int total = kCausal ? 0 : a.BH * nq;
  const int ntiles = kCausal ? ((nq - 1 - bx != bx) ? 2 : 1)
                             : (bx < total ? (total - 1 - bx) / static_cast<int>(gridDim.x) + 1 : 0);
  auto tile_unit = [&](int qt) { return bx + qt * static_cast<int>(gridDim.x); };
  auto tile_qb = [&](int qt) { return kCausal ? (qt == 0 ? nq - 1 - bx : bx) : tile_unit(qt) % nq; };
  auto tile_bh = [&](int qt) { return kCausal ? static_cast<int>(blockIdx.y) : tile_unit(qt) / nq; };
  auto tile_blocks = [&](int qt) { return kCausal ? min(nkv, tile_qb(qt) + 1) : nkv; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(s_free, 4);
    mbar_init(o_free, 4);
    mbar_init(&mma_done[0], 1);
    mbar_init(&mma_done[1], 1);
    if (kBiasTma) {
      for (int i = 0; i < 4; ++i) mbar_init(&turn[i], 1);
    }
    *abort_flag = 0;
    *never_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
    if (kBiasTma) tma_prefetch_desc(&tmB);
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
  DevStatus quiet = a.st;
  quiet.word = nullptr;
  if (warp < 4) {
    setmaxnreg_dec<Cfg::regs_low()>();
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ producer --
      int g = 0;        // K/V blocks issued
      int q_issued = 0;
      bool aborted = false;
      for (int qt = 0; qt < ntiles && !aborted; ++qt) {
        if (qt > 0 && !mbar_wait(q_empty, (qt - 1) & 1, abort_flag, a.st, 0x1104)) { aborted = true; break; }
        mbar_arrive_expect_tx(q_full, Cfg::kTileBytes);
#pragma unroll
        for (int c = 0; c < Cfg::kChunks; ++c) {
          tma_load_3d(sQ + c * 16384, &tmQ, q_full, c * 64, tile_qb(qt) * 128, tile_bh(qt));
        }
        q_issued = qt + 1;
        const int n = tile_blocks(qt);
        for (int j = 0; j < n; ++j, ++g) {
          const int s = g % KS;
          const uint32_t ph = (g / KS) & 1;
          if (!mbar_wait(&k_empty[s], ph ^ 1, abort_flag, a.st, 0x1100)) { aborted = true; break; }
          mbar_arrive_expect_tx(&k_full[s], Cfg::kTileBytes);
#pragma unroll
          for (int c = 0; c < Cfg::kChunks; ++c) {
            tma_load_3d(sK + s * Cfg::kTileBytes + c * 16384, &tmK, &k_full[s], c * 64, j * 128, tile_bh(qt));
          }
          if (!mbar_wait(&v_empty[s], ph ^ 1, abort_flag, a.st, 0x1101)) {
            mbar_wait(&k_full[s], ph, never_flag, quiet, 0);  // K is in flight; V is not
            aborted = true;
            break;
          }
          mbar_arrive_expect_tx(&v_full[s], Cfg::kTileBytes);
#pragma unroll
          for (int c = 0; c < Cfg::kChunks; ++c) {
            tma_load_3d(sV + s * Cfg::kTileBytes + c * 16384, &tmV, &v_full[s], c * 64, j * 128, tile_bh(qt));
          }
        }
      }
      if (aborted) {
        // Drain this CTA's own copies still in flight before it exits.
        if (q_issued > 0) mbar_wait(q_full, (q_issued - 1) & 1, never_flag, quiet, 0);
        for (int i = (g > KS ? g - KS : 0); i < g; ++i) {
          mbar_wait(&k_full[i % KS], (i / KS) & 1, never_flag, quiet, 0);
          mbar_wait(&v_full[i % KS], (i / KS) & 1, never_flag, quiet, 0);
        }
      }
    } else if (warp == 1 && lane == 0) {
      // -------------------------------------------------------- QK issuer --
      constexpr uint32_t idesc_qk = idesc_f16_f32(128, 128, 0, 0);
      const uint64_t q_desc0 = sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t k_desc0 = sdesc_sw128(smem_u32(sK), 16, 1024);
      int g = 0;
      bool ok_run = true;
      for (int qt = 0; qt < ntiles && ok_run; ++qt) {
        if (!mbar_wait(q_full, qt & 1, abort_flag, a.st, 0x1200)) break;
        const int n = tile_blocks(qt);
        for (int j = 0; j < n; ++j, ++g) {
          const int s = g % KS;
          if (!mbar_wait(&k_full[s], (g / KS) & 1, abort_flag, a.st, 0x1213)) { ok_run = false; break; }
          // S may be overwritten once the softmax holds the previous S in registers.
          if (g > 0 && !mbar_wait(s_free, (g - 1) & 1, abort_flag, a.st, 0x1218)) { ok_run = false; break; }
          tc_fence_after();
          const uint64_t kd = k_desc0 + static_cast<uint64_t>((s * Cfg::kTileBytes) >> 4);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t off = static_cast<uint64_t>(((k >> 2) * 16384 + (k & 3) * 32) >> 4);
            umma_f16_ss(tmem + Cfg::s_col(0), q_desc0 + off, kd + off, idesc_qk, k > 0 ? 1u : 0u);
          }
          umma_commit(s_full);
          umma_commit(&k_empty[s]);
        }
        if (ok_run) umma_commit(q_empty);  // Q buffer free once this tile's QKs finish
      }
      umma_commit(&mma_done[0]);
      mbar_wait(&mma_done[0], 0, never_flag, quiet, 0);
    } else if (warp == 3 && lane == 0) {
      // -------------------------------------------------------- PV issuer --
      constexpr uint32_t idesc_pv = idesc_f16_f32(128, D, 0, 1);
      const uint64_t v_desc0 = sdesc_sw128(smem_u32(sV), 16384, 1024);
      int g = 0;
      bool ok_run = true;
      for (int qt = 0; qt < ntiles && ok_run; ++qt) {
        const int n = tile_blocks(qt);
        for (int j = 0; j < n; ++j, ++g) {
          const int s = g % KS;
          if (!mbar_wait(&v_full[s], (g / KS) & 1, abort_flag, a.st, 0x1212)) { ok_run = false; break; }
          // The first PV of a tile overwrites O: the previous tile's epilogue must have read it.
          if (j == 0 && qt > 0 && !mbar_wait(o_free, (qt - 1) & 1, abort_flag, a.st, 0x1222)) { ok_run = false; break; }
          if (!mbar_wait(p_full, g & 1, abort_flag, a.st, 0x1210)) { ok_run = false; break; }
          tc_fence_after();
          const uint64_t vd = v_desc0 + static_cast<uint64_t>((s * Cfg::kTileBytes) >> 4);
          const uint32_t p_tmem = tmem + Cfg::p_col(0);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            umma_f16_ts(tmem + Cfg::o_col(0), p_tmem + (k >> 2) * Cfg::kPHalfStride + (k & 3) * 8,
                        vd + static_cast<uint64_t>((k * 2048) >> 4), idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(o_done);
          umma_commit(&v_empty[s]);
        }
      }
      umma_commit(&mma_done[1]);
      mbar_wait(&mma_done[1], 0, never_flag, quiet, 0);
    }
  } else {
    // ------------------------------------------------- softmax / epilogue --
    setmaxnreg_inc<kRegsHigh>();
    const int t = 0;
    const uint32_t q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((q * 32) << 16);
    const bool fast_path = a.qk_log2 > 0.f;
    const int ntile0 = 0, ntile1 = 0;  // turn handshake of the two-tile form: not used here
    (void)ntile0;
    (void)ntile1;
    bool ok_run = true;
    int g = 0;
    uint8_t* stage = sOut + (warp - 4) * kWarpBytes;
    // Dense bias: lane 0 requests the warp's 32 rows x 128 keys of key block
    // j of tile qt one block ahead, two 64-key boxes into `stage` (the
    // previous block's values are in registers by then).
    uint64_t* bias_full = &turn[q];
    int b_issued = 0;
    auto bias_issue = [&](int qt_, int j_) {
      const int y = tile_qb(qt_) * 128 + static_cast<int>(q) * 32;
      mbar_arrive_expect_tx(bias_full, 8192);
      tma_load_3d(stage, &tmB, bias_full, j_ * 128, y, tile_bh(qt_));
      tma_load_3d(stage + 4096, &tmB, bias_full, j_ * 128 + 64, y, tile_bh(qt_));
      ++b_issued;
    };
    if (kBiasTma && lane == 0 && ntiles > 0) bias_issue(0, 0);
    for (int qt = 0; qt < ntiles && ok_run; ++qt) {
      const int q0 = tile_qb(qt) * 128;
      const int bh = tile_bh(qt);
      const int h = bh % a.H;
      const int qrow = q0 + row;
      const int n_t = tile_blocks(qt);
      const float* ttab = kBias == kBiasTable ? a.table + static_cast<int64_t>(h) * (2 * S - 1) : nullptr;
      const int d0 = (qrow - lane) - 127 + S - 1;  // this warp's window start, block 0
      float* tb_win = tb_base + q * 160;
      float tpre[5];
      if (kBias == kBiasTable) table_window_load(tpre, ttab, d0, 2 * S - 1, static_cast<int>(lane));
      float m_used = -INFINITY;
      float l = 0.f;
      for (int j = 0; j < n_t; ++j, ++g) {
        // Warp-uniform: every lane must agree before the .sync.aligned TMEM ops.
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[t], g & 1, abort_flag, a.st, 0x1300 + t))) {
          ok_run = false;
          break;
        }
        tc_fence_after();
        float z[128];
        {
          // Four TMEM loads in flight, one wait.
          uint32_t r0[32], r1[32], r2[32], r3[32];
          tmem_ld32(lane_base + Cfg::s_col(t) + 0, r0);
          tmem_ld32(lane_base + Cfg::s_col(t) + 32, r1);
          tmem_ld32(lane_base + Cfg::s_col(t) + 64, r2);
          tmem_ld32(lane_base + Cfg::s_col(t) + 96, r3);
          tmem_wait_ld();
          if (!Cfg::kAliasP) {
            // S_t(j) is in registers: the issuer may compute S_t(j+1) now.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[t]);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            z[i] = __uint_as_float(r0[i]);
            z[32 + i] = __uint_as_float(r1[i]);
            z[64 + i] = __uint_as_float(r2[i]);
            z[96 + i] = __uint_as_float(r3[i]);
          }
        }
        const int k0 = j * 128;
        const bool edge = (k0 + 128 > S) || (kCausal && k0 + 127 > qrow);
        // Without a bias and with a positive scale, max(s) * c = max(s * c): the
        // row max is taken on the raw scores and each probability costs one FFMA
        // + one ex2. Otherwise z holds the log2-domain logits.
        // A dense bias is added to the raw scores (one mixed fp16 + fp32 add
        // per key, exact like converting first) and takes the same path.
        const bool raw_scores = (kBias != kBiasTable) && fast_path;
        if (kBias == kBiasDense) {
          if (!__all_sync(0xffffffffu, mbar_wait(bias_full, g & 1, abort_flag, a.st, 0x1330))) {
            ok_run = false;
            break;
          }
#pragma unroll
          for (int v = 0; v < 16; ++v) {
            // Key chunk v & 7 of row `lane` in box v >> 3, 128-byte swizzle:
            // the 8 lanes of a shared-memory phase hit 8 different chunks.
            const uint4 raw =
                *reinterpret_cast<const uint4*>(stage + (v >> 3) * 4096 + lane * 128 + (((v & 7) ^ (lane & 7)) << 4));
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              z[v * 8 + 2 * e] = add_f16_lo(w[e], z[v * 8 + 2 * e]);
              z[v * 8 + 2 * e + 1] = add_f16_hi(w[e], z[v * 8 + 2 * e + 1]);
            }
          }
          __syncwarp();
          if (lane == 0 && j + 1 < n_t) {
            fence_async_smem();  // the warp's reads of `stage` before the copy that overwrites it
            bias_issue(qt, j + 1);
          }
        } else if (kBias == kBiasTable) {
          const float* trow = table_window_store(tb_win, tpre, static_cast<int>(lane));
          if (j + 1 < n_t) table_window_load(tpre, ttab, d0 - 128 * (j + 1), 2 * S - 1, static_cast<int>(lane));
          const uint64_t qk2 = f2_pack(a.qk_log2, a.qk_log2);
#pragma unroll
          for (int col = 0; col < 128; col += 2) {
            const uint64_t r2 = ffma2(f2_pack(z[col], z[col + 1]), qk2, f2_pack(trow[-col], trow[-col - 1]));
            z[col] = f2_lo(r2);
            z[col + 1] = f2_hi(r2);
          }
        }
        if (kBias != kBiasTable && !raw_scores) {
#pragma unroll
          for (int col = 0; col < 128; ++col) z[col] *= a.qk_log2;
        }
        if (edge) {
#pragma unroll
          for (int col = 0; col < 128; ++col) {
            const int key = k0 + col;
            if (key >= S || (kCausal && key > qrow)) z[col] = -INFINITY;
          }
        }
        // Row max, 8 independent chains of 3-input max.
        float pm[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pm[i] = fmaxf(z[i], z[8 + i]);
#pragma unroll
        for (int c = 16; c < 128; c += 16) {
#pragma unroll
          for (int i = 0; i < 8; ++i) pm[i] = fmax3(pm[i], z[c + i], z[c + 8 + i]);
        }
        float rmax = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                           fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
        if (raw_scores) rmax *= a.qk_log2;
        const float m_new = fmaxf(m_used, rmax);
        const bool need = m_new > m_used + kRescaleThreshold;
        float alpha = 1.f;
        if (need) {
          alpha = ex2_approx(m_used - m_new);
          m_used = m_new;
        }
        const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
        const float zc = raw_scores ? a.qk_log2 : 1.f;
        // Ping-pong on the exp unit: the two warps that share this SM
        // sub-partition (same lane quarter q, tiles 0 and 1) take strict turns
        // for their exp loops, tile 0 first. Everything else a tile does (TMEM
        // traffic, row max, P store, its MMAs) then hides under the other
        // tile's exps instead of both tiles stalling at the same time.
        // Tile 0 block j waits for tile 1's block j-1 (when tile 1 exists);
        // tile 1 block j waits for tile 0's block j (an existing tile 1 never
        // has fewer blocks than tile 0).
        const bool wait_turn = kT == 2 && ((t == 0) ? (j > 0 && ntile1 > 0) : (j < ntile0));
        if (wait_turn) {
          const uint32_t par = (t == 0) ? ((j - 1) & 1) : (j & 1);
          if (!__all_sync(0xffffffffu, mbar_wait(&turn[t * 4 + q], par, abort_flag, a.st, 0x1340 + t))) {
            ok_run = false;
            break;
          }
        }
        // p = 2^(z * zc - m), one ex2 per element, fp32 row sums in 8
        // partials; the exponent arguments and the sums are formed two
        // lanes per instruction (packed fp32 FMA / add).
        float ps[8];
        uint32_t pk[64];
        const uint64_t zc2 = f2_pack(zc, zc);
        const uint64_t nm2 = f2_pack(neg_m, neg_m);
        uint64_t acc2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const uint64_t x2 = ffma2(f2_pack(z[2 * i], z[2 * i + 1]), zc2, nm2);
          const float p0 = ex2_approx(f2_lo(x2));
          const float p1 = ex2_approx(f2_hi(x2));
          acc2[i & 3] = fadd2(acc2[i & 3], f2_pack(p0, p1));
          pk[i] = pack_half2(p0, p1);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          ps[2 * i] = f2_lo(acc2[i]);
          ps[2 * i + 1] = f2_hi(acc2[i]);
        }
        const float sum = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
        // Hand the exp unit to the partner warp of the other tile.
        if (kT == 2) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&turn[(1 - t) * 4 + q]);
        }
        if (!Cfg::kAliasP && j > 0) {
          // P_t and O_t are still in use by PV_t(j-1) until it completes.
          if (!__all_sync(0xffffffffu, mbar_wait(&o_done[t], (g - 1) & 1, abort_flag, a.st, 0x1320 + t))) {
            ok_run = false;
            break;
          }
          tc_fence_after();
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t q16[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) q16[i] = pk[c * 16 + i];
          tmem_st16(lane_base + Cfg::p_col(t) + c * 16, q16);
        }
        l = l * alpha + sum;
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // PV_t(j-1) is complete (waited on above, or implied by s_full when P
          // aliases S).
          uint32_t r[32];
  #pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            tmem_ld32(lane_base + Cfg::o_col(t) + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(lane_base + Cfg::o_col(t) + c * 32, r);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      if (!ok_run) break;
      // ----------------------------------------------------------- epilogue --
      if (!__all_sync(0xffffffffu, mbar_wait(o_done, (g - 1) & 1, abort_flag, a.st, 0x1310))) {
        ok_run = false;
        break;
      }
      tc_fence_after();
      const float inv_l = 1.f / l;
      const int row0 = q0 + static_cast<int>(q) * 32;
      constexpr int kStores = D / 32;  // fp32: 32 columns per store; fp16: 64
      const int nst = a.out_f16 ? kStores / 2 : kStores;
#pragma unroll 1
      for (int c = 0; c < nst; ++c) {
        uint32_t w[32];
        if (a.out_f16) {
          uint32_t r0[32], r1[32];
          tmem_ld32(lane_base + Cfg::o_col(0) + c * 64, r0);
          tmem_ld32(lane_base + Cfg::o_col(0) + c * 64 + 32, r1);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            w[i] = pack_half2(__uint_as_float(r0[2 * i]) * inv_l, __uint_as_float(r0[2 * i + 1]) * inv_l);
            w[16 + i] = pack_half2(__uint_as_float(r1[2 * i]) * inv_l, __uint_as_float(r1[2 * i + 1]) * inv_l);
          }
        } else {
          uint32_t r[32];
          tmem_ld32(lane_base + Cfg::o_col(0) + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(__uint_as_float(r[i]) * inv_l);
        }
        if (c == nst - 1) {
          // O is in registers: the next tile's first PV may overwrite it.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(o_free);
        }
        if (lane == 0) bulk_wait_read_all();  // the previous store has read the staging rows
        __syncwarp();
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          *reinterpret_cast<uint4*>(stage + lane * 128 + ((v ^ (lane & 7)) << 4)) =
              make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0 && row0 < S) {
          tma_store_3d(&tmO, stage, c * (a.out_f16 ? 64 : 32), row0, bh);
          bulk_commit();
        }
      }
      if (kBiasTma && lane == 0 && qt + 1 < ntiles) {
        bulk_wait_read_all();  // the O stores have read the staging rows
        bias_issue(qt + 1, 0);
      }
    }
    if (kBiasTma && lane == 0 && b_issued > g) {
      // Left early with the next block's bias in flight: let it land first.
      mbar_wait(bias_full, (b_issued - 1) & 1, never_flag, quiet, 0);
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// One work unit = (query block of 256 rows, batch*head). Units are walked
// heaviest first when causal, and grouped by head otherwise so the CTAs that
// run at the same time share K/V in L2.
__device__ __forceinline__ void unit_coords(int w, int nqb, int BH, bool causal, int& qb, int& bh) {
  if (causal) {
    qb = nqb - 1 - w / BH;
    bh = w % BH;
  } else {
    bh = w / nqb;
    qb = w % nqb;
  }
}

// Unit k of this CTA as published by the producer (-1: no more units; -2:
// the wait was abandoned); counts the caller as one of the slot's readers.
__device__ __noinline__ int fetch_unit(uint64_t* full, uint64_t* empty, volatile int* ring, int k,
                                       volatile int* abort_flag, DevStatus st) {
  if (!mbar_wait(&full[k % kUnitRing], (k / kUnitRing) & 1, abort_flag, st, 0x1401)) return -2;
  const int w = ring[k % kUnitRing];
  mbar_arrive(&empty[k % kUnitRing]);
  return w;
}

// Persistent variant of the kernel above: one CTA per SM walks work units
// until a per-launch ticket counter runs past the last one. The producer
// takes the tickets and publishes each unit index in a small smem ring
// (unit_full / unit_empty) that every other role reads in the same order, so
// a CTA's prologue (barrier init, TMEM allocation) is paid once per SM and an
// SM that runs faster takes more units. Every mbarrier phase is tracked with
// running counters across units; o_free[t] lets the first PV of the next unit
// overwrite O_t only after the epilogue has read it, and the exp-unit turn
// handshake continues across unit boundaries.
template <int D, bool kCausal, int kBias>
__global__ void __launch_bounds__(FaCfg<D>::kThreads, 1)
    fa2_persistent_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV,
                          const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmB,
                          FaArgs a) {
  using Cfg = FaCfg<D>;
  constexpr int KS = Cfg::kStages;
  constexpr int QB = Cfg::kQBuffers;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // QB x (2 tiles)
  uint8_t* sK = smem + QB * 2 * Cfg::kTileBytes;        // KS tiles
  uint8_t* sV = sK + KS * Cfg::kTileBytes;              // KS tiles
  uint8_t* sOut = sV + KS * Cfg::kTileBytes;          // 4 KB per softmax warp
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + Cfg::kOutBytes);
  uint64_t* q_full = bars;              // [QB]
  uint64_t* q_empty = q_full + QB;      // [QB] last QK of the unit done
  uint64_t* k_full = q_empty + QB;      // [KS]
  uint64_t* k_empty = k_full + KS;
  uint64_t* v_full = k_empty + KS;
  uint64_t* v_empty = v_full + KS;
  uint64_t* s_full = v_empty + KS;      // [2]
  uint64_t* p_full = s_full + 2;        // [2]
  uint64_t* o_done = p_full + 2;        // [2]
  uint64_t* s_free = o_done + 2;        // [2] softmax has read S_t (4 warps)
  uint64_t* o_free = s_free + 2;        // [2] epilogue has read O_t (4 warps)
  uint64_t* mma_done = o_free + 2;      // [2] [0]: the MMA issuer's last MMAs done ([1] unused)
  uint64_t* turn = mma_done + 2;        // [2][4] exp-loop turn of tile t, lane quarter q
  uint64_t* unit_full = turn + 8;       // [kUnitRing] unit index published
  uint64_t* unit_empty = unit_full + kUnitRing;  // [kUnitRing] read by all consumers
  volatile int* unit_ring = reinterpret_cast<volatile int*>(unit_empty + kUnitRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(unit_empty + kUnitRing) + kUnitRing;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* never_flag = abort_flag + 1;  // stays 0: drain waits ignore the abort

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int S = a.S;
  const int nkv = (S + 127) / 128;
  const int num_units = a.num_qblocks * a.BH;
  // KV blocks each Q tile of unit (q0) visits (0 for a tile that starts past S)
  auto ntile = [&](int q0, int t) {
    const int start = q0 + 128 * t;
    return start >= S ? 0 : (kCausal ? min(nkv, start / 128 + 1) : nkv);
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < QB; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_done[t], 1);
      mbar_init(&s_free[t], 4);
      mbar_init(&o_free[t], 4);
      mbar_init(&mma_done[t], 1);
    }
    for (int i = 0; i < 8; ++i) mbar_init(&turn[i], 1);
    for (int i = 0; i < kUnitRing; ++i) {
      mbar_init(&unit_full[i], 1);
      mbar_init(&unit_empty[i], kUnitReaders);
    }
    *abort_flag = 0;
    *never_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
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
  DevStatus quiet = a.st;
  quiet.word = nullptr;
  // Unit k of this CTA for a single-thread consumer (see fetch_unit).
  auto take_unit = [&](int k) -> int {
    if (!mbar_wait(&unit_full[k % kUnitRing], (k / kUnitRing) & 1, abort_flag, a.st, 0x1400)) return -2;
    const int w = unit_ring[k % kUnitRing];
    mbar_arrive(&unit_empty[k % kUnitRing]);
    return w;
  };

  if (warp < 4) {
    // Warpgroup 0: TMA producer, MMA issuer, TMEM allocator.
    setmaxnreg_dec<kRegsLowPersistent>();
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ producer --
      int g = 0;
      int q_issued = 0;
      bool aborted = false;
      // Units are handed out dynamically: the first one by block index, the
      // rest from a per-launch counter, so SMs that run faster take more.
      int w = blockIdx.x;
      for (int k = 0; !aborted; ++k) {
        if (!mbar_wait(&unit_empty[k % kUnitRing], ((k / kUnitRing) & 1) ^ 1, abort_flag, a.st, 0x1103)) {
          aborted = true;
          break;
        }
        unit_ring[k % kUnitRing] = w < num_units ? w : -1;
        mbar_arrive(&unit_full[k % kUnitRing]);
        if (w >= num_units) break;
        const int w_next = static_cast<int>(gridDim.x) + atomicAdd(a.unit_counter, 1);
        int qb, bh;
        unit_coords(w, a.num_qblocks, a.BH, kCausal, qb, bh);
        const int q0 = qb * 256;
        const int n0 = ntile(q0, 0), n1 = ntile(q0, 1), nmax = max(n0, n1);
        const int qi = k % QB;
        if (!mbar_wait(&q_empty[qi], ((k / QB) & 1) ^ 1, abort_flag, a.st, 0x1102)) { aborted = true; break; }
        mbar_arrive_expect_tx(&q_full[qi], (n1 > 0 ? 2 : 1) * Cfg::kTileBytes);
        for (int t = 0; t < 2; ++t) {
          if ((t ? n1 : n0) == 0) continue;
#pragma unroll
          for (int c = 0; c < Cfg::kChunks; ++c) {
            tma_load_3d(sQ + (qi * 2 + t) * Cfg::kTileBytes + c * 16384, &tmQ, &q_full[qi], c * 64, q0 + 128 * t, bh);
          }
        }
        q_issued = k + 1;
        for (int j = 0; j < nmax; ++j, ++g) {
          const int s = g % KS;
          const uint32_t ph = (g / KS) & 1;
          if (!mbar_wait(&k_empty[s], ph ^ 1, abort_flag, a.st, 0x1100)) { aborted = true; break; }
          mbar_arrive_expect_tx(&k_full[s], Cfg::kTileBytes);
#pragma unroll
          for (int c = 0; c < Cfg::kChunks; ++c) {
            tma_load_3d(sK + s * Cfg::kTileBytes + c * 16384, &tmK, &k_full[s], c * 64, j * 128, bh);
          }
          if (!mbar_wait(&v_empty[s], ph ^ 1, abort_flag, a.st, 0x1101)) {
            mbar_wait(&k_full[s], ph, never_flag, quiet, 0);  // K_j is in flight; V_j is not
            aborted = true;
            break;
          }
          mbar_arrive_expect_tx(&v_full[s], Cfg::kTileBytes);
#pragma unroll
          for (int c = 0; c < Cfg::kChunks; ++c) {
            tma_load_3d(sV + s * Cfg::kTileBytes + c * 16384, &tmV, &v_full[s], c * 64, j * 128, bh);
          }
        }
        w = w_next;
      }
      if (aborted) {
        // Drain this CTA's own copies still in flight before it exits.
        for (int i = (q_issued > QB ? q_issued - QB : 0); i < q_issued; ++i) {
          mbar_wait(&q_full[i % QB], (i / QB) & 1, never_flag, quiet, 0);
        }
        for (int i = (g > KS ? g - KS : 0); i < g; ++i) {
          mbar_wait(&k_full[i % KS], (i / KS) & 1, never_flag, quiet, 0);
          mbar_wait(&v_full[i % KS], (i / KS) & 1, never_flag, quiet, 0);
        }
      }
    } else if (warp == 1 && lane == 0) {
      // ------------------------------------------------------- MMA issuer --
      // One thread issues both tiles' MMAs in the order S_t(0) = Q_t K(0)^T,
      // then per key block j: O_t += P_t(j) V(j) followed at once by
      // S_t(j+1) = Q_t K(j+1)^T. P_t lives in S_t's columns; tcgen05.mma
      // operations from one thread execute in issue order, so the QK that
      // overwrites S_t runs after the PV that reads P_t without waiting for
      // that PV to complete (a wait on its commit, then a second thread's
      // issue, sat in every tile's chain before). s_full_t(j+1) completing
      // also means PV_t(j) has, which is what the softmax needs before it
      // rescales O_t.
      constexpr uint32_t idesc_qk = idesc_f16_f32(128, 128, 0, 0);
      constexpr uint32_t idesc_pv = idesc_f16_f32(128, D, 0, 1);
      // Descriptor bases, computed once; a K step only moves the start
      // address field (low bits), so the per-MMA work is one 64-bit add.
      const uint64_t q_desc0 = sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t k_desc0 = sdesc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t v_desc0 = sdesc_sw128(smem_u32(sV), 16384, 1024);
      // pph bits 0-1: parity of the P blocks tile 0/1 has had; bits 2-3:
      // parity of the units tile 0/1 has finished; bits 4-5: tile 0/1 has
      // finished a unit (its O buffer has an epilogue to wait for).
      uint32_t pph = 0;
      int ks = 0, vs = 0;            // K and V stages
      uint32_t kph = 0, vph = 0;     // their phases
      bool ok_run = true;
      auto issue_qk = [&](int t, int qi) {
        const uint64_t qd = q_desc0 + static_cast<uint64_t>(((qi * 2 + t) * Cfg::kTileBytes) >> 4);
        const uint64_t kd = k_desc0 + static_cast<uint64_t>((ks * Cfg::kTileBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = static_cast<uint64_t>(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
          umma_f16_ss(tmem + Cfg::s_col(t), qd + off, kd + off, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto next_k = [&]() {
        umma_commit(&k_empty[ks]);
        if (++ks == KS) { ks = 0; kph ^= 1u; }
      };
      for (int k = 0; ok_run; ++k) {
        const int w = take_unit(k);
        if (w < 0) break;
        int qb, bh;
        unit_coords(w, a.num_qblocks, a.BH, kCausal, qb, bh);
        const int q0 = qb * 256;
        const int n0 = ntile(q0, 0), n1 = ntile(q0, 1), nmax = max(n0, n1);
        const int qi = QB == 1 ? 0 : (k & 1);
        if (!mbar_wait(&q_full[qi], (k / QB) & 1, abort_flag, a.st, 0x1200)) break;
        if (nmax > 0) {
          if (!mbar_wait(&k_full[ks], kph, abort_flag, a.st, 0x1213)) break;
          tc_fence_after();
          if (n0 > 0) issue_qk(0, qi);
          if (n1 > 0) issue_qk(1, qi);
          next_k();
        }
        // The Q buffer is free once this unit's last QKs finish: release it
        // as soon as they are issued, so the next unit's Q load starts under
        // this unit's last softmax blocks.
        if (nmax <= 1) umma_commit(&q_empty[qi]);
        for (int j = 0; ok_run && j < nmax; ++j) {
          if (!mbar_wait(&v_full[vs], vph, abort_flag, a.st, 0x1212)) { ok_run = false; break; }
          if (j + 1 < nmax && !mbar_wait(&k_full[ks], kph, abort_flag, a.st, 0x1213)) { ok_run = false; break; }
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (j >= (t ? n1 : n0)) continue;
            if (j == 0 && (pph & (16u << t))) {
              // The first PV of a unit overwrites O_t: the previous unit's
              // epilogue must have read it.
              if (!mbar_wait(&o_free[t], ((pph >> (2 + t)) & 1u) ^ 1u, abort_flag, a.st, 0x1222 + t)) {
                ok_run = false;
                break;
              }
            }
            if (!mbar_wait(&p_full[t], (pph >> t) & 1u, abort_flag, a.st, 0x1210 + t)) { ok_run = false; break; }
            tc_fence_after();
            const uint64_t vd = v_desc0 + static_cast<uint64_t>((vs * Cfg::kTileBytes) >> 4);
            const uint32_t p_tmem = tmem + Cfg::p_col(t);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              umma_f16_ts(tmem + Cfg::o_col(t), p_tmem + (kk >> 2) * Cfg::kPHalfStride + (kk & 3) * 8,
                          vd + static_cast<uint64_t>((kk * 2048) >> 4), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(&o_done[t]);
            pph ^= 1u << t;
            if (j + 1 < (t ? n1 : n0)) issue_qk(t, qi);
          }
          if (!ok_run) break;
          umma_commit(&v_empty[vs]);
          if (++vs == KS) { vs = 0; vph ^= 1u; }
          if (j + 1 < nmax) next_k();
          if (j + 2 == nmax) umma_commit(&q_empty[qi]);  // the unit's last QKs are issued
        }
        if (!ok_run) break;
        if (n0 > 0) pph = (pph ^ 4u) | 16u;
        if (n1 > 0) pph = (pph ^ 8u) | 32u;
      }
      // Every MMA this thread issued must be complete before TMEM is freed.
      umma_commit(&mma_done[0]);
      mbar_wait(&mma_done[0], 0, never_flag, quiet, 0);
    }
  } else {
    // ------------------------------------------------- softmax / epilogue --
    setmaxnreg_inc<kRegsHighPersistent>();
    const int t = (warp - 4) >> 2;
    const uint32_t q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((q * 32) << 16);
    const bool fast_path = a.qk_log2 > 0.f;
    bool ok_run = true;
    // Phase word, kept in one register across units: bit 0 = parity of the
    // blocks this tile has handled (s_full; o_done of the previous block is
    // its complement), bit 1 = parity of the turns this warp has waited for,
    // bit 2 = the previous unit had a tile 1 (tile 0 only).
    uint32_t ph = 0;
    for (int k = 0; ok_run; ++k) {
      // Lane 0 takes the unit for the warp. The wait sits in a call so the
      // register allocation of the softmax loop below does not have to keep
      // the wait loop's state.
      int w = -2;
      if (lane == 0) w = fetch_unit(unit_full, unit_empty, unit_ring, k, abort_flag, a.st);
      w = __shfl_sync(0xffffffffu, w, 0);
      if (w < 0) break;
      int qb, bh;
      unit_coords(w, a.num_qblocks, a.BH, kCausal, qb, bh);
      const int q0 = qb * 256;
      const int n_t = ntile(q0, t);
      const int partner = ntile(q0, 1 - t);  // blocks of the other tile
      const bool first_wait = (ph & 4u) != 0;
      if (t == 0) ph = (ph & ~4u) | (partner > 0 ? 4u : 0u);
      if (n_t == 0) continue;
      const int qrow = q0 + 128 * t + row;
      const int h = bh % a.H;
      const float* ttab = kBias == kBiasTable ? a.table + static_cast<int64_t>(h) * (2 * S - 1) : nullptr;
      const int d0 = (qrow - lane) - 127 + S - 1;  // this warp's window start, block 0
      float* tb_win = reinterpret_cast<float*>(sOut + (warp - 4) * 4096);  // in this warp's O staging block
      float tpre[5];
      if (kBias == kBiasTable) table_window_load(tpre, ttab, d0, 2 * S - 1, static_cast<int>(lane));
      const __half* brow = nullptr;
      if (kBias == kBiasDense) brow = a.bias + bh * a.bias_head + static_cast<int64_t>(min(qrow, S - 1)) * a.bias_row;
      float m_used = -INFINITY;
      float l = 0.f;
      for (int j = 0; j < n_t; ++j, ph ^= 1u) {
        // Dense bias: this row's 128 values of block j are requested before
        // the wait for S, so their latency hides under the QK MMA.
        uint4 braw[kBias == kBiasDense ? 16 : 1];
        if (kBias == kBiasDense) {
#pragma unroll
          for (int v = 0; v < 16; ++v) {
            const int key = j * 128 + v * 8;
            braw[v] = key + 8 <= S ? __ldg(reinterpret_cast<const uint4*>(brow + key)) : make_uint4(0, 0, 0, 0);
          }
        }
        // Warp-uniform: every lane must agree before the .sync.aligned TMEM ops.
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[t], ph & 1u, abort_flag, a.st, 0x1300 + t))) {
          ok_run = false;
          break;
        }
        tc_fence_after();
        float z[128];
        {
          // Four TMEM loads in flight, one wait.
          uint32_t r0[32], r1[32], r2[32], r3[32];
          tmem_ld32(lane_base + Cfg::s_col(t) + 0, r0);
          tmem_ld32(lane_base + Cfg::s_col(t) + 32, r1);
          tmem_ld32(lane_base + Cfg::s_col(t) + 64, r2);
          tmem_ld32(lane_base + Cfg::s_col(t) + 96, r3);
          tmem_wait_ld();
          if (!Cfg::kAliasP) {
            // S_t is in registers: the issuer may compute the next S_t now.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[t]);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            z[i] = __uint_as_float(r0[i]);
            z[32 + i] = __uint_as_float(r1[i]);
            z[64 + i] = __uint_as_float(r2[i]);
            z[96 + i] = __uint_as_float(r3[i]);
          }
        }
        const int k0 = j * 128;
        const bool edge = (k0 + 128 > S) || (kCausal && k0 + 127 > qrow);
        // Without a bias and with a positive scale, max(s) * c = max(s * c): the
        // row max is taken on the raw scores and each probability costs one FFMA
        // + one ex2. Otherwise z holds the log2-domain logits.
        // A dense bias is added to the raw scores (one mixed fp16 + fp32 add
        // per key, exact like converting first) and takes the same path.
        const bool raw_scores = (kBias != kBiasTable) && fast_path;
        if (kBias == kBiasDense) {
#pragma unroll
          for (int v = 0; v < 16; ++v) {
            const uint32_t w[4] = {braw[v].x, braw[v].y, braw[v].z, braw[v].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              z[v * 8 + 2 * e] = add_f16_lo(w[e], z[v * 8 + 2 * e]);
              z[v * 8 + 2 * e + 1] = add_f16_hi(w[e], z[v * 8 + 2 * e + 1]);
            }
          }
        } else if (kBias == kBiasTable) {
          if (j == 0) {
            // The window shares this warp's O staging block: the previous unit's
            // stores must have read it.
            if (lane == 0) bulk_wait_read_all();
          }
          const float* trow = table_window_store(tb_win, tpre, static_cast<int>(lane));
          if (j + 1 < n_t) table_window_load(tpre, ttab, d0 - 128 * (j + 1), 2 * S - 1, static_cast<int>(lane));
          const uint64_t qk2 = f2_pack(a.qk_log2, a.qk_log2);
#pragma unroll
          for (int col = 0; col < 128; col += 2) {
            const uint64_t r2 = ffma2(f2_pack(z[col], z[col + 1]), qk2, f2_pack(trow[-col], trow[-col - 1]));
            z[col] = f2_lo(r2);
            z[col + 1] = f2_hi(r2);
          }
        }
        if (kBias != kBiasTable && !raw_scores) {
#pragma unroll
          for (int col = 0; col < 128; ++col) z[col] *= a.qk_log2;
        }
        if (edge) {
#pragma unroll
          for (int col = 0; col < 128; ++col) {
            const int key = k0 + col;
            if (key >= S || (kCausal && key > qrow)) z[col] = -INFINITY;
          }
        }
        // Row max, 8 independent chains of 3-input max.
        float pm[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pm[i] = fmaxf(z[i], z[8 + i]);
#pragma unroll
        for (int c = 16; c < 128; c += 16) {
#pragma unroll
          for (int i = 0; i < 8; ++i) pm[i] = fmax3(pm[i], z[c + i], z[c + 8 + i]);
        }
        float rmax = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                           fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
        if (raw_scores) rmax *= a.qk_log2;
        const float m_new = fmaxf(m_used, rmax);
        const bool need = m_new > m_used + kRescaleThreshold;
        float alpha = 1.f;
        if (need) {
          alpha = ex2_approx(m_used - m_new);
          m_used = m_new;
        }
        const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
        const float zc = raw_scores ? a.qk_log2 : 1.f;
        // Ping-pong on the exp unit: the two warps that share this SM
        // sub-partition (same lane quarter q, tiles 0 and 1) take strict turns
        // for their exp loops. Over the CTA's units the exp loops form one
        // sequence 0_0 1_0 0_1 1_1 ... (tile 1 may have one block more, or
        // none); a loop waits for the partner when the item before it in that
        // sequence is the partner's, and arrives when the item after it is
        // (tile 1's last block always arrives: if no unit follows, that phase
        // is simply never waited for). Each turn barrier thus completes one
        // phase per wait and never runs two phases ahead of its waiter.
        const bool wait_turn = (t == 0) ? (j > 0 ? partner > 0 : first_wait) : (j < partner);
        if (wait_turn) {
          if (!__all_sync(0xffffffffu, mbar_wait(&turn[t * 4 + q], (ph >> 1) & 1u, abort_flag, a.st, 0x1340 + t))) {
            ok_run = false;
            break;
          }
          ph ^= 2u;
        }
        // p = 2^(z * zc - m), one ex2 per element, fp32 row sums in 8
        // partials; the exponent arguments and the sums are formed two
        // lanes per instruction (packed fp32 FMA / add).
        float ps[8];
        uint32_t pk[64];
        const uint64_t zc2 = f2_pack(zc, zc);
        const uint64_t nm2 = f2_pack(neg_m, neg_m);
        uint64_t acc2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const uint64_t x2 = ffma2(f2_pack(z[2 * i], z[2 * i + 1]), zc2, nm2);
          const float p0 = ex2_approx(f2_lo(x2));
          const float p1 = ex2_approx(f2_hi(x2));
          acc2[i & 3] = fadd2(acc2[i & 3], f2_pack(p0, p1));
          pk[i] = pack_half2(p0, p1);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          ps[2 * i] = f2_lo(acc2[i]);
          ps[2 * i + 1] = f2_hi(acc2[i]);
        }
        const float sum = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
        // Hand the exp unit to the partner warp when its loop comes next.
        if (t == 0 ? (partner > 0)
                   : (j + 1 < partner || j + 1 == n_t)) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&turn[(1 - t) * 4 + q]);
        }
        if (!Cfg::kAliasP && j > 0) {
          // P_t and O_t are still in use by the previous PV until it completes
          // (for j == 0 the previous unit's epilogue already waited for it).
          if (!__all_sync(0xffffffffu, mbar_wait(&o_done[t], (ph & 1u) ^ 1u, abort_flag, a.st, 0x1320 + t))) {
            ok_run = false;
            break;
          }
          tc_fence_after();
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t q16[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) q16[i] = pk[c * 16 + i];
          tmem_st16(lane_base + Cfg::p_col(t) + c * 16, q16);
        }
        l = l * alpha + sum;
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // The previous PV is complete (waited on above, or implied by s_full
          // when P aliases S).
          uint32_t r[32];
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            tmem_ld32(lane_base + Cfg::o_col(t) + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(lane_base + Cfg::o_col(t) + c * 32, r);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      if (!ok_run) break;
      // ----------------------------------------------------------- epilogue --
      if (!__all_sync(0xffffffffu, mbar_wait(&o_done[t], (ph & 1u) ^ 1u, abort_flag, a.st, 0x1310 + t))) {
        ok_run = false;
        break;
      }
      tc_fence_after();
      const float inv_l = 1.f / l;
      // 32 rows x 128 bytes per TMA store through this warp's 128-byte-swizzled
      // staging rows; rows past S are clipped by the store.
      uint8_t* stage = sOut + (warp - 4) * 4096;
      const int row0 = q0 + 128 * t + static_cast<int>(q) * 32;
      constexpr int kStores = D / 32;  // fp32: 32 columns per store; fp16: 64
#pragma unroll 1
      for (int c = 0; c < (a.out_f16 ? kStores / 2 : kStores); ++c) {
        uint32_t w[32];
        const bool last_ld = c == (a.out_f16 ? kStores / 2 : kStores) - 1;
        if (a.out_f16) {
          uint32_t r0[32], r1[32];
          tmem_ld32(lane_base + Cfg::o_col(t) + c * 64, r0);
          tmem_ld32(lane_base + Cfg::o_col(t) + c * 64 + 32, r1);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            w[i] = pack_half2(__uint_as_float(r0[2 * i]) * inv_l, __uint_as_float(r0[2 * i + 1]) * inv_l);
            w[16 + i] = pack_half2(__uint_as_float(r1[2 * i]) * inv_l, __uint_as_float(r1[2 * i + 1]) * inv_l);
          }
        } else {
          uint32_t r[32];
          tmem_ld32(lane_base + Cfg::o_col(t) + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(__uint_as_float(r[i]) * inv_l);
        }
        if (last_ld) {
          // O_t is in registers: the next unit's first PV may overwrite it.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[t]);
        }
        if (lane == 0) bulk_wait_read_all();  // the previous store has read the staging rows
        __syncwarp();
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          *reinterpret_cast<uint4*>(stage + lane * 128 + ((v ^ (lane & 7)) << 4)) =
              make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0 && row0 < S) {
          tma_store_3d(&tmO, stage, c * (a.out_f16 ? 64 : 32), row0, bh);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  if (threadIdx.x == 0) {
    // Thread 0 took this CTA's last ticket above; once every CTA has counted
    // itself out nobody reads the counter again in this launch.
    __threadfence();
    if (atomicAdd(a.unit_counter + 1, 1) == static_cast<int>(gridDim.x) - 1) {
      atomicExch(a.unit_counter, 0);
      atomicExch(a.unit_counter + 1, 0);
    }
  }
}

struct FaProblem {
  const void *Q, *K, *V;
  int64_t q_row, q_head, k_row, k_head, v_row, v_head;  // elements
  void* O;
  int64_t o_row, o_head;
  bool out_f16;
  int BH, H, S, D;
  float scale;
  bool causal;
  int bias_mode;
  const float* table;
  const void* bias;
  int64_t bias_head, bias_row;
};

template <class Kernel>
int run_fa2_kernel(Kernel kern, int threads, uint32_t regs_low, uint32_t regs_high, dim3 grid, int smem_bytes,
                   const CUtensorMap& tq,
                   const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& to, const CUtensorMap& tb, const FaArgs& args,
                   cudaStream_t stream) {
  cudaFuncAttributes fa{};
  int rc = kernel_setup(reinterpret_cast<const void*>(kern), smem_bytes, &fa);
  if (rc != NESO_OK) return rc;
  if (static_cast<int64_t>(fa.numRegs) * threads < 128 * regs_low + (threads - 128) * regs_high) {
    return fail(NESO_ERR_LAUNCH, "fa2: %d registers/thread cannot fund the %u/%u warpgroup split", fa.numRegs,
                regs_low, regs_high);
  }
  cudaError_t e = launch_pdl(kern, grid, dim3(threads), smem_bytes, stream, tq, tk, tv, to, tb, args);
  if (e != cudaSuccess) return cuda_fail(e, "fa2 launch");
  return ok();
}

// Kernel per head dim, the faster one measured on B200: D = 128 runs the
// persistent two-tile kernel, D = 64 the one-tile CTA walking its tiles
// (persistent when non-causal, tiles qb and nq-1-qb when causal).
template <int D, bool kCausal, int kBias>
int launch_fa2_t(const FaProblem& p, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                 const CUtensorMap& to, const CUtensorMap& tb, FaArgs& args, cudaStream_t stream) {
  using Cfg = FaCfg<D>;
  if constexpr (D == 128) {
    const int units = args.num_qblocks * p.BH;
    int rc = stream_counters(stream, &args.unit_counter);
    if (rc != NESO_OK) return rc;
    return run_fa2_kernel(fa2_persistent_kernel<D, kCausal, kBias>, Cfg::kThreads, kRegsLowPersistent, kRegsHighPersistent,
                          dim3(units < sm_count() ? units : sm_count(), 1, 1), Cfg::kSmemBytes, tq, tk, tv, to, tb,
                          args, stream);
  } else {
    // 128-row units, two CTAs per SM.
    using Cfg1 = FaCfg<D, 1>;
    constexpr int smem = pair_smem_bytes<D, kBias>();
    args.num_qblocks = (p.S + 127) / 128;
    if constexpr (kCausal) {
      // Causal: tiles qb and nq-1-qb share a CTA (nq + 1 key blocks each CTA).
      return run_fa2_kernel(fa2_pair_kernel<D, kCausal, kBias>, Cfg1::kThreads, Cfg1::regs_low(), kRegsHigh,
                            dim3((args.num_qblocks + 1) / 2, p.BH, 1), smem, tq, tk, tv, to, tb, args, stream);
    } else {
      // Persistent: two CTAs per SM walk the (head, query tile) units.
      const int64_t total = static_cast<int64_t>(args.num_qblocks) * p.BH;
      const int grid = static_cast<int>(std::min<int64_t>(total, 2 * static_cast<int64_t>(sm_count())));
      return run_fa2_kernel(fa2_pair_kernel<D, kCausal, kBias>, Cfg1::kThreads, Cfg1::regs_low(), kRegsHigh, dim3(grid, 1, 1),
                            smem, tq, tk, tv, to, tb, args, stream);
    }
  }
}

template <int D>
int launch_fa2_d(const FaProblem& p, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                 const CUtensorMap& to, const CUtensorMap& tb, FaArgs& args, cudaStream_t stream) {
  if (p.causal) {
    if (p.bias_mode == kBiasTable) return launch_fa2_t<D, true, kBiasTable>(p, tq, tk, tv, to, tb, args, stream);
    if (p.bias_mode == kBiasDense) return launch_fa2_t<D, true, kBiasDense>(p, tq, tk, tv, to, tb, args, stream);
    return launch_fa2_t<D, true, kBiasNone>(p, tq, tk, tv, to, tb, args, stream);
  }
  if (p.bias_mode == kBiasTable) return launch_fa2_t<D, false, kBiasTable>(p, tq, tk, tv, to, tb, args, stream);
  if (p.bias_mode == kBiasDense) return launch_fa2_t<D, false, kBiasDense>(p, tq, tk, tv, to, tb, args, stream);
  return launch_fa2_t<D, false, kBiasNone>(p, tq, tk, tv, to, tb, args, stream);
}

int make_qkv_map(CUtensorMap* m, const void* base, int D, int S, int BH, int64_t row, int64_t head) {
  uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(S), static_cast<uint64_t>(BH)};
  uint64_t strides[2] = {static_cast<uint64_t>(row) * 2, static_cast<uint64_t>(head) * 2};
  uint32_t box[3] = {64, 128, 1};
  return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int launch_fa2(const FaProblem& p, cudaStream_t stream) {
  if (p.D != 64 && p.D != 128) return fail(NESO_ERR_UNSUPPORTED, "head dim %d not supported (64 or 128)", p.D);
  if (p.S <= 0 || p.BH <= 0) return ok();
  if (p.Q == nullptr || p.K == nullptr || p.V == nullptr || p.O == nullptr) {
    return fail(NESO_ERR_INVALID_ARG, "null Q/K/V/O pointer");
  }
  if (p.q_row < p.D || p.k_row < p.D || p.v_row < p.D || p.o_row < p.D) {
    return fail(NESO_ERR_INVALID_ARG, "row stride smaller than the head dim");
  }
  if ((reinterpret_cast<uintptr_t>(p.O) & 15u) != 0 || (p.o_row % 8) != 0 || (p.o_head % 8) != 0) {
    return fail(NESO_ERR_MISALIGNED, "O must be 16-byte aligned with row/head strides multiple of 8 elements");
  }
  if (p.bias_mode == kBiasDense &&
      ((reinterpret_cast<uintptr_t>(p.bias) & 15u) != 0 || p.bias_row % 8 != 0 || p.bias_head % 8 != 0)) {
    return fail(NESO_ERR_MISALIGNED, "bias must be 16-byte aligned with strides multiple of 8 elements");
  }
  if (p.bias_mode == kBiasTable && p.table == nullptr) return fail(NESO_ERR_INVALID_ARG, "null table");
  if (p.bias_mode == kBiasDense && p.bias == nullptr) return fail(NESO_ERR_INVALID_ARG, "null bias");
  CUtensorMap tq, tk, tv;
  int rc = make_qkv_map(&tq, p.Q, p.D, p.S, p.BH, p.q_row, p.q_head);
  if (rc == NESO_OK) rc = make_qkv_map(&tk, p.K, p.D, p.S, p.BH, p.k_row, p.k_head);
  if (rc == NESO_OK) rc = make_qkv_map(&tv, p.V, p.D, p.S, p.BH, p.v_row, p.v_head);
  if (rc != NESO_OK) return rc;
  // O as [BH][S][D] for TMA stores (the alignment checks above make its
  // strides multiples of 16 bytes): boxes of 32 rows x 128 bytes.
  CUtensorMap to;
  {
    const int esz = p.out_f16 ? 2 : 4;
    uint64_t dims[3] = {static_cast<uint64_t>(p.D), static_cast<uint64_t>(p.S), static_cast<uint64_t>(p.BH)};
    uint64_t strides[2] = {static_cast<uint64_t>(p.o_row) * esz, static_cast<uint64_t>(p.o_head) * esz};
    uint32_t box[3] = {static_cast<uint32_t>(128 / esz), 32, 1};
    rc = encode_tmap(&to, p.out_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, p.O, dims,
                     strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NESO_OK) return rc;
  }
  // Dense bias as [BH][S rows][S keys] for the one-tile kernel's TMA loads:
  // boxes of 32 rows x 64 keys (128 bytes); keys and rows past S read 0.
  CUtensorMap tb = to;
  if (p.bias_mode == kBiasDense && p.D == 64) {
    uint64_t dims[3] = {static_cast<uint64_t>(p.S), static_cast<uint64_t>(p.S), static_cast<uint64_t>(p.BH)};
    uint64_t strides[2] = {static_cast<uint64_t>(p.bias_row) * 2, static_cast<uint64_t>(p.bias_head) * 2};
    uint32_t box[3] = {64, 32, 1};
    rc = encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, p.bias, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NESO_OK) return rc;
  }
  FaArgs args{};
  args.O = p.O;
  args.o_row = p.o_row;
  args.o_head = p.o_head;
  args.S = p.S;
  args.H = p.H;
  args.qk_log2 = p.scale * kLog2e;
  args.table = p.table;
  args.bias = static_cast<const __half*>(p.bias);
  args.bias_head = p.bias_head;
  args.bias_row = p.bias_row;
  args.num_qblocks = (p.S + 255) / 256;
  args.BH = p.BH;
  args.unit_counter = nullptr;
  args.out_f16 = p.out_f16 ? 1 : 0;
  rc = device_status(&args.st);
  if (rc != NESO_OK) return rc;
  if (p.D == 64) return launch_fa2_d<64>(p, tq, tk, tv, to, tb, args, stream);
  return launch_fa2_d<128>(p, tq, tk, tv, to, tb, args, stream);
}

// The reference's BM is a compile-time tile height (8..128, power of two);
// its grid is (N / BM, ...). Accept exactly those grids.
int check_ref_grid_x(uint32_t gx, int N) {
  if (gx == 0 || N % static_cast<int>(gx) != 0) {
    return fail(NESO_ERR_GRID, "grid_x=%u does not divide N=%d (reference grid is (N/BM, ...))", gx, N);
  }
  const int bm = N / static_cast<int>(gx);
  if (bm < 8 || bm > 128 || (bm & (bm - 1)) != 0) {
    return fail(NESO_ERR_GRID, "grid_x=%u implies BM=%d; the reference BM is a power of two in [8,128]", gx, bm);
  }
  return NESO_OK;
}

// The hand-written MSL kernels (bench/bench_flash_attention.py:142-149,
// bench/bench_flash_attention_opt.py:145-152, bench/bench_fa2_d128.py:116-123)
// take Q, K, V and O in one `io_type` (half or float) with d_head and scale as
// runtime constants. fp32 operands are rounded to fp16 for the tensor cores
// (three [N, d] copies in the stream's input workspace); O stays in io_type.
__global__ void f32_to_f16_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                  const float* __restrict__ c, __half* __restrict__ out, int64_t n) {
  const bool vec = n % 4 == 0 && ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                                   reinterpret_cast<uintptr_t>(c)) & 15u) == 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int t = 0; t < 3; ++t) {
    const float* src = t == 0 ? a : (t == 1 ? b : c);
    __half* dst = out + t * n;
    if (vec) {
      for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n / 4; i += stride) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(src) + i);
        __half2* d2 = reinterpret_cast<__half2*>(dst + 4 * i);
        d2[0] = __floats2half2_rn(v.x, v.y);
        d2[1] = __floats2half2_rn(v.z, v.w);
      }
    } else {
      for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
        dst[i] = __float2half_rn(__ldg(src + i));
      }
    }
  }
}

int fa2_msl(const void* Q, const void* K, const void* V, void* O, int32_t N, int32_t d_head, float scale,
            int32_t BM, int32_t BN, int32_t d, int32_t THREADS, int32_t use_half, uint32_t gx, uint32_t gy,
            uint32_t gz, cudaStream_t stream, int only_d) {
  if (BM <= 0 || BN <= 0 || THREADS <= 0) return fail(NESO_ERR_INVALID_ARG, "BM, BN and THREADS must be positive");
  if (use_half != 0 && use_half != 1) return fail(NESO_ERR_INVALID_ARG, "use_half must be 0 or 1");
  if (d != 64 && d != 128) return fail(NESO_ERR_UNSUPPORTED, "head dim d=%d not supported (64 or 128)", d);
  if (only_d != 0 && d != only_d) return fail(NESO_ERR_UNSUPPORTED, "this kernel is compiled for d=%d", only_d);
  if (d_head != d) return fail(NESO_ERR_INVALID_ARG, "d_head=%d differs from the kernel's d=%d", d_head, d);
  if (N <= 0) return fail(NESO_ERR_INVALID_ARG, "N must be positive");
  if (N % BM != 0 || gx != static_cast<uint32_t>(N / BM) || gy != 1 || gz != 1) {
    return fail(NESO_ERR_GRID, "grid (%u,%u,%u) != (N/BM, 1, 1) with N=%d BM=%d (N a multiple of BM)", gx, gy, gz, N,
                BM);
  }
  if (Q == nullptr || K == nullptr || V == nullptr || O == nullptr) {
    return fail(NESO_ERR_INVALID_ARG, "null Q/K/V/O pointer");
  }
  FaProblem p{};
  p.Q = Q; p.K = K; p.V = V; p.O = O;
  p.q_row = p.k_row = p.v_row = p.o_row = d;
  p.q_head = p.k_head = p.v_head = p.o_head = static_cast<int64_t>(N) * d;
  p.out_f16 = use_half != 0;
  p.BH = 1; p.H = 1; p.S = N; p.D = d;
  p.scale = scale;
  p.causal = false;
  p.bias_mode = kBiasNone;
  if (!use_half) {
    const int64_t n = static_cast<int64_t>(N) * d;
    void* ws = nullptr;
    int rc = stream_workspace(stream, static_cast<size_t>(3 * n) * sizeof(__half), &ws, kWorkspaceInputs);
    if (rc != NESO_OK) return rc;
    __half* h = static_cast<__half*>(ws);
    const int blocks = static_cast<int>(std::min<int64_t>((n / 4 + 255) / 256 + 1, 4 * sm_count()));
    f32_to_f16_kernel<<<blocks, 256, 0, stream>>>(static_cast<const float*>(Q), static_cast<const float*>(K),
                                                  static_cast<const float*>(V), h, n);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "fp32 -> fp16 operand launch");
    p.Q = h; p.K = h + n; p.V = h + 2 * n;
  }
  return launch_fa2(p, stream);
}

}  // namespace
}  // namespace neso

using namespace neso;

extern "C" {

int neso_flash_attention_fwd(const void* Q, const void* K, const void* V, float* O, int32_t N, int32_t stride_qo,
                             int32_t stride_kv, float scale, int32_t HEAD_DIM, uint32_t grid_x, uint32_t grid_y,
                             uint32_t grid_z, neso_stream_t stream) {
  if (N <= 0) return fail(NESO_ERR_INVALID_ARG, "N must be positive");
  int rc = check_ref_grid_x(grid_x, N);
  if (rc != NESO_OK) return rc;
  if (grid_y != 1 || grid_z != 1) return fail(NESO_ERR_GRID, "single-head FA2 grid must be (N/BM, 1, 1)");
  FaProblem p{};
  p.Q = Q; p.K = K; p.V = V; p.O = O;
  p.q_row = stride_qo; p.k_row = stride_kv; p.v_row = stride_kv; p.o_row = stride_qo;
  p.q_head = static_cast<int64_t>(stride_qo) * N;
  p.k_head = static_cast<int64_t>(stride_kv) * N;
  p.v_head = p.k_head;
  p.o_head = p.q_head;
  p.out_f16 = false;
  p.BH = 1; p.H = 1; p.S = N; p.D = HEAD_DIM;
  p.scale = scale;
  p.causal = false;
  p.bias_mode = kBiasNone;
  return launch_fa2(p, as_stream(stream));
}

int neso_rel_pos_fa2_fwd(const void* Q, const void* K, const void* V, const void* bias, void* O, int32_t T,
                         int32_t stride, float scale, int32_t stride_h, int32_t bias_stride_h, int32_t HEAD_DIM,
                         uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream) {
  if (T <= 0) return fail(NESO_ERR_INVALID_ARG, "T must be positive");
  int rc = check_ref_grid_x(grid_x, T);
  if (rc != NESO_OK) return rc;
  if (grid_y == 0 || grid_z != 1) return fail(NESO_ERR_GRID, "rel-pos FA2 grid must be (T/BM, nh, 1)");
  if (static_cast<int64_t>(bias_stride_h) < static_cast<int64_t>(T) * T) {
    return fail(NESO_ERR_INVALID_ARG, "bias_stride_h %d < T*T", bias_stride_h);
  }
  FaProblem p{};
  p.Q = Q; p.K = K; p.V = V; p.O = O;
  p.q_row = p.k_row = p.v_row = p.o_row = stride;
  p.q_head = p.k_head = p.v_head = p.o_head = stride_h;
  p.out_f16 = true;
  p.BH = static_cast<int>(grid_y); p.H = p.BH; p.S = T; p.D = HEAD_DIM;
  p.scale = scale;
  p.causal = false;
  p.bias_mode = kBiasDense;
  p.bias = bias;
  p.bias_head = bias_stride_h;
  p.bias_row = T;
  return launch_fa2(p, as_stream(stream));
}

int neso_fa2_fwd(const void* Q, const void* K, const void* V, float* O, int32_t B, int32_t H, int32_t S, int32_t D,
                 float scale, int32_t causal, neso_stream_t stream) {
  if (B < 0 || H < 0 || S < 0) return fail(NESO_ERR_INVALID_ARG, "negative size");
  if (static_cast<int64_t>(B) * H > 65535) return fail(NESO_ERR_UNSUPPORTED, "B*H must be <= 65535");
  FaProblem p{};
  p.Q = Q; p.K = K; p.V = V; p.O = O;
  p.q_row = p.k_row = p.v_row = p.o_row = D;
  p.q_head = p.k_head = p.v_head = p.o_head = static_cast<int64_t>(S) * D;
  p.out_f16 = false;
  p.BH = B * H; p.H = H; p.S = S; p.D = D;
  p.scale = scale;
  p.causal = causal != 0;
  p.bias_mode = kBiasNone;
  return launch_fa2(p, as_stream(stream));
}

int neso_fa2_fwd_relpos_table(const void* Q, const void* K, const void* V, const float* table, float* O, int32_t B,
                              int32_t H, int32_t S, int32_t D, float scale, int32_t causal, neso_stream_t stream) {
  if (B < 0 || H < 0 || S < 0) return fail(NESO_ERR_INVALID_ARG, "negative size");
  if (static_cast<int64_t>(B) * H > 65535) return fail(NESO_ERR_UNSUPPORTED, "B*H must be <= 65535");
  FaProblem p{};
  p.Q = Q; p.K = K; p.V = V; p.O = O;
  p.q_row = p.k_row = p.v_row = p.o_row = D;
  p.q_head = p.k_head = p.v_head = p.o_head = static_cast<int64_t>(S) * D;
  p.out_f16 = false;
  p.BH = B * H; p.H = H; p.S = S; p.D = D;
  p.scale = scale;
  p.causal = causal != 0;
  p.bias_mode = kBiasTable;
  p.table = table;
  return launch_fa2(p, as_stream(stream));
}

int neso_flash_attention_fwd_msl(const void* Q, const void* K, const void* V, void* O, int32_t N, int32_t d_head,
                                 float scale, int32_t BM, int32_t BN, int32_t d, int32_t THREADS, int32_t use_half,
                                 uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream) {
  return fa2_msl(Q, K, V, O, N, d_head, scale, BM, BN, d, THREADS, use_half, grid_x, grid_y, grid_z,
                 as_stream(stream), 0);
}

int neso_flash_attention_opt(const void* Q, const void* K, const void* V, void* O, int32_t N, int32_t d_head,
                             float scale, int32_t BM, int32_t BN, int32_t d, int32_t THREADS, int32_t use_half,
                             uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream) {
  return fa2_msl(Q, K, V, O, N, d_head, scale, BM, BN, d, THREADS, use_half, grid_x, grid_y, grid_z,
                 as_stream(stream), 0);
}

int neso_flash_attention_d128(const void* Q, const void* K, const void* V, void* O, int32_t N, int32_t d_head,
                              float scale, int32_t BM, int32_t BN, int32_t d, int32_t THREADS, int32_t use_half,
                              uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream) {
  return fa2_msl(Q, K, V, O, N, d_head, scale, BM, BN, d, THREADS, use_half, grid_x, grid_y, grid_z,
                 as_stream(stream), 128);
}

}  // extern "C"
