// Flash-attention forward for NVIDIA B200 (sm_100a).
//
// Computes O = softmax(scale * Q K^T) V for fp16 [B,H,S,D] tensors, the
// operation of the reference's HIP kernels (attn_kernel.hip:146-708) behind its
// C-ABI `launch` (attn_kernel.hip:710-742). The algorithm is the same tiled
// online softmax: K/V are streamed in key tiles, each query row keeps a running
// max m and running sum l, partial outputs are rescaled by exp(m_old - m_new)
// when the max grows (attn_kernel.hip:452-462, 491-492), and the output is
// O / l at the end (attn_kernel.hip:497-511). The S x S score matrix is never
// written to memory.
//
// The B200 design (attn_fwd_kernel, head dim <= 128):
//  * Persistent CTAs, one per SM, walk a list of units; a unit is two 128-row
//    query tiles of one (batch, head), multiplied against every 128-key K/V
//    tile, so each K/V tile is read from L2 once per 256 query rows. The key
//    range of the last, partial wave of units can be split across CTAs, with
//    the partial results combined on the GPU (SegIter, make_plan).
//  * A producer warp streams each unit's Q and the K/V tiles (a ring of
//    shared-memory stages, one key tile's K and V per stage) with TMA,
//    128-byte swizzled, completion tracked by mbarriers.
//  * The MMA warp issues every tcgen05.mma (four per elected lane): S_i =
//    Q_i K^T (fp16 x fp16 -> fp32, both operands from shared memory) into
//    tensor memory (TMEM), and O_i += P_i V with P_i read from TMEM and V from
//    shared memory.
//  * Two softmax warpgroups (one per query tile, one thread per query row =
//    one TMEM lane) read S_i from TMEM, update m and l in fp32, write
//    P_i = exp2(S_i * scale * log2(e) - m) as fp16 back into the S_i columns of
//    TMEM, and rescale their O_i rows in TMEM when the max grows by more than
//    2^8 (otherwise the stale max is kept: O and l carry the same factor, so
//    O / l is unchanged, and P stays <= 256).
//  * The MMA order S0(j), PV1(j-1), S1(j), PV0(j) lets softmax 0 run while the
//    tensor core works on tile 1 and vice versa.
//  * D <= 64: P_i has TMEM columns of its own, and S_i(j+1) is issued as soon
//    as the first half of P_i(j) is published (by then the softmax holds all
//    of S_i(j) in registers), so the next S no longer waits for the PV that
//    reads P. Per key tile: PV0(j) keys 0-63, S0(j+1), PV0(j) keys 64-127,
//    the same for tile 1; the softmax waits for PV_i(j-1) before its first
//    P store and O rescale.
//  * Epilogue: O_i / l -> fp16, each warp's 32 rows staged in 4 KiB of shared
//    memory and stored as whole 128-byte row segments (a split piece writes
//    unnormalised fp32 O, m and l to the workspace instead; the last piece
//    combines them and stores the same way).
//
// TMEM columns (512 allocated): S0 [0,128), S1 [128,256), O0 [256,256+DP),
// O1 [256+DP, 256+2*DP). At D = 128 P_i occupies the first 64 columns of S_i;
// at D <= 64 P0 is [384,448) and P1 [448,512).
//
// Every mbarrier wait is bounded (time limit from the host). A wait that runs
// out sets a CTA-wide abort flag and the device status word, the other roles
// stop at their next wait, in-flight copies and MMAs are drained with bounded
// waits, TMEM is freed and the kernel returns.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <mutex>

#include "../../include/gfx906_b200_attn.h"
#include "sm100_ptx.cuh"

namespace fa {

constexpr int BM = 128;            // query rows per tile (= TMEM lanes)
constexpr int BN = 128;            // keys per K/V tile
constexpr int CHUNK_BYTES = 16384; // one 128-row x 64-col fp16 swizzled box
constexpr int NUM_THREADS = 384;   // 2 softmax warpgroups + 1 control warpgroup
// Register split after launch (launch: 384 x 168 = 64512): the softmax
// warpgroups hold a 128-column score row per thread; the control warpgroup
// (producer, MMA issuer, two idle warps) needs fewer. 256*200 + 128*96 = 63488.
constexpr uint32_t REGS_SOFTMAX = 200;
constexpr uint32_t REGS_CONTROL = 96;
constexpr int PRODUCER_WARP = 8;
constexpr int MMA_WARP = 9;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units
constexpr int MAX_PIECES = 32;             // most pieces one split unit is cut into
#ifndef ATTN_EMU_PAIRS
#define ATTN_EMU_PAIRS 1
#endif
// Pairs of exponentials, out of every 4 pairs (8 columns), evaluated with the
// FMA-pipe polynomial instead of MUFU ex2 (balances the two pipes).
constexpr int EMU_PAIRS = ATTN_EMU_PAIRS;

// Roles recorded in the timeout diagnostics.
enum Role : int { ROLE_PRODUCER = 1, ROLE_MMA = 2, ROLE_SOFTMAX0 = 3, ROLE_SOFTMAX1 = 4 };

// Device status word: bit 0 = a bounded wait ran out. Sticky until the host
// clears it through gfx906_b200_attn_device_status(1).
__device__ unsigned int g_status = 0;
__device__ int g_timeout_info[6];

struct Params {
  int Sq;
  int Skv;
  int D;            // true head dim (<= DP)
  int bh_offset;    // added to blockIdx.y (D = 512 kernel)
  float scale_log2; // scale * log2(e)
  unsigned long long timeout_ns;
  // persistent schedule of attn_fwd_kernel
  int n_qb;               // query blocks (units) per (batch, head)
  int unit_rows;          // query rows per unit: 256 (two query tiles) or 128 (one)
  int n_units;            // n_qb * B * H
  int n_tiles;            // 128-key tiles per unit
  int split;              // 1: whole units, then a stream-K split of the tail units
  int tail_unit0;         // first unit of the split tail (split mode)
  int tail_ctas;          // CTAs that share the tail's key range (split mode)
  long long total_steps;  // (n_units - tail_unit0) * n_tiles: steps of the tail
  __half* o;              // output, [B*H, Sq, D] fp16
  float* ws_o;            // split workspace: [tail_ctas][2][2] slots of [DP/4][128][4] partial O
  float* ws_ml;           // [tail_ctas][2][2][128][2] partial (m, l)
  int combine;            // 1: the last piece of a unit combines it in the kernel (D <= 128)
  unsigned long long* ws_cnt;  // [tail units][2] arrival counters: (epoch << 8) | arrivals (combine == 1)
  unsigned long long epoch;    // unique per launch (56 bits), tags the counters
};

template <int DP>
struct Cfg {
  static constexpr int NCHUNK = DP / 64;
  static constexpr int TILE_BYTES = NCHUNK * CHUNK_BYTES;
  // Q buffers (2 lets the next unit's Q load during the current unit) and K/V
  // tile slots. Measured on B200: at DP=128 a second Q buffer, which leaves
  // room for only 3 slots, lost 2-5%; at DP=64 it made no difference.
  static constexpr int QBUFS = 1;
  static constexpr int STAGES = (DP == 128) ? 4 : 8;  // TILE_BYTES slots
  // The ring holds PAIRS key tiles: K(j) in slot 2p, V(j) in slot 2p+1, with
  // one full and one empty barrier per pair (one wait and one release per key
  // tile in the MMA warp, whose issue loop is on the critical path: measured
  // 2-6% faster than separate K and V barriers).
  static constexpr int PAIRS = STAGES / 2;
  // DP = 64 leaves 128 TMEM columns free (S0 S1 O0 O1 take 384): P then gets
  // columns of its own, [384, 448) and [448, 512), instead of overwriting S,
  // and the next S of a query tile no longer waits for the PV that reads P.
  static constexpr bool SEP_P = DP == 64;
  static constexpr uint32_t P_COL = 384;
  // barrier indices
  static constexpr int B_Q_FULL = 0;   // [2], per Q buffer
  static constexpr int B_Q_EMPTY = 2;  // [2]
  static constexpr int B_KV_FULL = 4;  // [PAIRS] used
  static constexpr int B_KV_EMPTY = 4 + STAGES;
  static constexpr int B_S_FULL = 4 + 2 * STAGES;
  static constexpr int B_P_FULL = B_S_FULL + 2;
  static constexpr int B_P_HALF = B_P_FULL + 2;  // [2]: first half of P stored
  static constexpr int B_O_FULL = B_P_HALF + 2;
  static constexpr int B_PV_DONE = B_O_FULL + 2;  // [2]: PV(j) done, P columns free (DP = 64)
  static constexpr int B_WG = B_PV_DONE + 2;  // per-warpgroup rendezvous, 2 barriers
  static constexpr int B_DRAIN = B_WG + 2;
  static constexpr int NUM_BARS = B_DRAIN + 1;
  static constexpr int DATA_BYTES = (2 * QBUFS + STAGES) * TILE_BYTES;
  // Output staging: 4 KiB per softmax warp (32 rows x 64 fp16 columns).
  static constexpr int EPI_OFF = (DATA_BYTES + NUM_BARS * 8 + 32 + 127) & ~127;
  static constexpr int SMEM_BYTES = 1024 /*alignment slack*/ + EPI_OFF + 8 * 4096;
};

__device__ __forceinline__ bool wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                       unsigned long long timeout_ns, int bar_idx, int role) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t n = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if ((++n & 31u) == 0u) {
      const uint64_t t = globaltimer_ns();
      if (t - t0 > timeout_ns || n > (1u << 24)) {
        *abort_flag = 1;
        if (atomicCAS(&g_status, 0u, 1u) == 0u) {
          g_timeout_info[0] = blockIdx.x;
          g_timeout_info[1] = blockIdx.y;
          g_timeout_info[2] = threadIdx.x / 32;
          g_timeout_info[3] = bar_idx;
          g_timeout_info[4] = static_cast<int>(parity);
          g_timeout_info[5] = role;
          __threadfence();
        } else {
          atomicOr(&g_status, 1u);
        }
        return false;
      }
    }
  }
}

// Bounded wait for completion of the phase with the given parity.
__device__ __forceinline__ bool bwait(uint32_t bars, int idx, uint32_t parity,
                                      volatile int* abort_flag, unsigned long long timeout_ns,
                                      int role) {
  const uint32_t bar = bars + 8u * idx;
  if (mbar_try_wait(bar, parity)) return true;
  return wait_slow(bar, parity, abort_flag, timeout_ns, idx, role);
}

// Warp-uniform bounded wait: every lane gets the same answer, so the
// warp-collective tcgen05.ld/st that follow are never reached by part of a warp.
__device__ __forceinline__ bool bwait_warp(uint32_t bars, int idx, uint32_t parity,
                                           volatile int* abort_flag, unsigned long long timeout_ns,
                                           int role) {
  const bool ok = bwait(bars, idx, parity, abort_flag, timeout_ns, role);
  return __all_sync(0xffffffffu, ok);
}

// Output rows through shared memory. A softmax thread owns one row of O;
// stored straight from registers, each warp store instruction would touch 32
// rows, i.e. 32 different 128-byte lines (measured on B200: ~5000 cycles per
// unit for the C2 epilogue). Instead each warp writes its 32 rows x 64
// columns as fp16 into its own 4 KiB staging tile (128-byte rows, 16-byte
// chunks XOR-swizzled by row: conflict-free both ways), then reads it back
// so that 8 lanes store one 128-byte row segment, 4 rows per instruction.
// stage_32 writes columns [32 cc, 32 cc + 32) of the tile for this lane's row.
__device__ __forceinline__ void stage_32(uint32_t stg, int lane, int cc, const uint32_t* o, float inv) {
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int ch = cc * 4 + e;
    st_shared_v4(stg + lane * 128 + ((ch ^ (lane & 7)) << 4),
                 pack_half2(__uint_as_float(o[8 * e + 0]) * inv, __uint_as_float(o[8 * e + 1]) * inv),
                 pack_half2(__uint_as_float(o[8 * e + 2]) * inv, __uint_as_float(o[8 * e + 3]) * inv),
                 pack_half2(__uint_as_float(o[8 * e + 4]) * inv, __uint_as_float(o[8 * e + 5]) * inv),
                 pack_half2(__uint_as_float(o[8 * e + 6]) * inv, __uint_as_float(o[8 * e + 7]) * inv));
  }
}
// Stores the warp's staged tile: rows row0 .. row0 + 31 (of Sq) of matrix
// base, columns [c0, c0 + 64) (of D; D % 8 == 0).
__device__ __forceinline__ void flush_stage(uint32_t stg, int lane, __half* base, int row0, int Sq, int D,
                                            int c0) {
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + (lane >> 3), ch = lane & 7;
    const uint4 v = ld_shared_v4(stg + r * 128 + ((ch ^ (r & 7)) << 4));
    const int col = c0 + ch * 8;
    if (row0 + r < Sq && col < D)
      *reinterpret_cast<uint4*>(base + static_cast<long long>(row0 + r) * D + col) = v;
  }
  __syncwarp();
}

// Max over the valid columns of a raw score row (min when the scale is
// negative), so that extreme * scale is the row max of the scaled scores.
__device__ __forceinline__ float row_extreme(const uint32_t* s, int nvalid, bool full, bool pos) {
  if (full) {
    float a0 = __uint_as_float(s[0]), a1 = __uint_as_float(s[1]);
    float a2 = __uint_as_float(s[2]), a3 = __uint_as_float(s[3]);
    if (pos) {
#pragma unroll
      for (int c = 4; c < BN; c += 8) {
        a0 = fmax3(a0, __uint_as_float(s[c]), __uint_as_float(s[c + 1]));
        a1 = fmax3(a1, __uint_as_float(s[c + 2]), __uint_as_float(s[c + 3]));
        if (c + 4 < BN) {
          a2 = fmax3(a2, __uint_as_float(s[c + 4]), __uint_as_float(s[c + 5]));
          a3 = fmax3(a3, __uint_as_float(s[c + 6]), __uint_as_float(s[c + 7]));
        }
      }
      return fmax3(fmaxf(a0, a1), a2, a3);
    }
#pragma unroll
    for (int c = 4; c < BN; c += 8) {
      a0 = fmin3(a0, __uint_as_float(s[c]), __uint_as_float(s[c + 1]));
      a1 = fmin3(a1, __uint_as_float(s[c + 2]), __uint_as_float(s[c + 3]));
      if (c + 4 < BN) {
        a2 = fmin3(a2, __uint_as_float(s[c + 4]), __uint_as_float(s[c + 5]));
        a3 = fmin3(a3, __uint_as_float(s[c + 6]), __uint_as_float(s[c + 7]));
      }
    }
    return fmin3(fminf(a0, a1), a2, a3);
  }
  float a0 = pos ? -INFINITY : INFINITY;
#pragma unroll
  for (int c = 0; c < BN; ++c) {
    const float x = __uint_as_float(s[c]);
    if (c < nvalid) a0 = pos ? fmaxf(a0, x) : fminf(a0, x);
  }
  return a0;
}

// P = exp2(s * sl2 + neg_m) for one 128-column score row, rounded to fp16 and
// stored into TMEM columns [tS, tS + 64) (two fp16 per column); returns the
// fp32 row sum in two partial sums. EMU_PAIRS of every 4 column pairs use the
// FMA-pipe polynomial, the rest MUFU. MASK zeroes columns >= nvalid (last
// key tile).
// When half_bar is non-zero, the first half of P (keys 0..63) is published on
// it as soon as it is stored (after before_half() has run), so the tensor core
// can start on those keys while the second half is computed. before_store()
// runs once, after the first half's exponentials and before any of P is stored.
template <bool MASK, typename BeforeHalf, typename BeforeStore>
__device__ __forceinline__ void row_exp_store(const uint32_t* s, float sl2, float neg_m, int nvalid,
                                              uint32_t tS, float& sum0, float& sum1, uint32_t half_bar,
                                              BeforeHalf&& before_half, BeforeStore&& before_store) {
  const uint64_t sl2x2 = f2_pack(sl2, sl2);
  const uint64_t negm2 = f2_pack(neg_m, neg_m);
  uint64_t acc0 = f2_pack(0.f, 0.f), acc1 = acc0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t pk[32];
#pragma unroll
    for (int c2 = 0; c2 < 32; ++c2) {
      const int c = h * 64 + 2 * c2;
      const uint64_t X = f2_fma(f2_pack(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), sl2x2, negm2);
      float x0, x1, e0, e1;
      f2_unpack(X, x0, x1);
      if ((c2 & 3) < EMU_PAIRS) {
        exp2_poly3_x2(x0, x1, e0, e1);
      } else {
        e0 = ex2_approx(x0);
        e1 = ex2_approx(x1);
      }
      if (MASK) {
        e0 = (c < nvalid) ? e0 : 0.f;
        e1 = (c + 1 < nvalid) ? e1 : 0.f;
      }
      if (c2 & 1)
        acc1 = f2_add(acc1, f2_pack(e0, e1));
      else
        acc0 = f2_add(acc0, f2_pack(e0, e1));
      pk[c2] = pack_half2(e0, e1);
    }
    if (h == 0) before_store();
    tmem_st32(tS + 32 * h, pk);
    if (h == 0 && half_bar) {
      before_half();
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(half_bar);
    }
  }
  float a, b, c, d;
  f2_unpack(acc0, a, b);
  f2_unpack(acc1, c, d);
  sum0 = a + c;
  sum1 = b + d;
}

// Multiply this thread's TMEM row of O (DP fp32 columns at tO) by factor when
// do_it (warp-uniform).
template <int DP>
__device__ __forceinline__ void rescale_rows(uint32_t tO, bool do_it, float factor) {
  if (!do_it) return;
#pragma unroll
  for (int c = 0; c < DP / 16; ++c) {
    uint32_t o[16];
    tmem_ld16(tO + 16 * c, o);
    tmem_wait_ld();
    reg_fence16(o);
#pragma unroll
    for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
    tmem_st16(tO + 16 * c, o);
  }
}

// Persistent schedule shared by every role of attn_fwd_kernel: a CTA walks a
// list of segments (unit, first key tile, end key tile). A unit is one
// 256-row query block of one (batch, head) -- 128 rows (one query tile) for
// problems too small to fill half the SMs otherwise. CTA c first takes whole units c,
// c+G, c+2G, ... below tail_unit0 (all units in whole mode). In split mode the
// remaining "tail" units are then shared by the first tail_ctas CTAs: CTA c
// owns the contiguous range [c*W/tail_ctas, (c+1)*W/tail_ctas) of the tail's
// W = units * key-tiles steps, so the machine stays balanced to one key tile;
// a tail unit whose key range spans several CTAs is computed as partial
// pieces, combined by the last one to finish. Partials only ever occur at the
// end of a CTA's work.
struct SegIter {
  long long s, s_end;
  int u, G, T, tail0;
  bool first_tail;
  __device__ __forceinline__ void init(const Params& p, int c, int G_) {
    G = G_;
    T = p.n_tiles;
    u = c;
    tail0 = p.split ? p.tail_unit0 : p.n_units;
    s = s_end = 0;
    if (p.split && c < p.tail_ctas) {
      s = static_cast<long long>(c) * p.total_steps / p.tail_ctas;
      s_end = static_cast<long long>(c + 1) * p.total_steps / p.tail_ctas;
    }
    first_tail = true;
  }
  // first_seg: this is the CTA's first tail segment (selects its partial slot).
  __device__ __forceinline__ bool next(int& unit, int& t0, int& t1, bool& first_seg) {
    if (u < tail0) {
      unit = u;
      t0 = 0;
      t1 = T;
      u += G;
      first_seg = false;
      return true;
    }
    if (s >= s_end) return false;
    const int rel = static_cast<int>(s / T);
    unit = tail0 + rel;
    const long long ubase = static_cast<long long>(rel) * T;
    const long long e = (s_end < ubase + T) ? s_end : ubase + T;
    t0 = static_cast<int>(s - ubase);
    t1 = static_cast<int>(e - ubase);
    s = e;
    first_seg = first_tail;
    first_tail = false;
    return true;
  }
};

__device__ __forceinline__ long long range_begin(long long W, int G, int c) {
  return static_cast<long long>(c) * W / G;
}
// Index of the CTA whose step range contains `step` (split mode). Range c
// starts at floor(c * W / G), so "range c+1 starts at or before step" is
// (c+1) * W < (step+1) * G: one division for the estimate, none to correct it.
__device__ __forceinline__ int owner_cta(long long step, long long W, int G) {
  int c = static_cast<int>((step * G) / W);
  const long long lim = (step + 1) * G;
  while (c + 1 < G && static_cast<long long>(c + 1) * W < lim) ++c;
  while (c > 0 && static_cast<long long>(c) * W >= lim) --c;
  return c;
}

template <int DP>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const Params p) {
  using C = Cfg<DP>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t s0 = (raw + 1023u) & ~1023u;  // 1024-B aligned for the 128B swizzle
  uint8_t* smem = smem_raw + (s0 - raw);
  const uint32_t sQ = s0;  // Q buffer b, query tile i at sQ + (2 * b + i) * TILE_BYTES
  const uint32_t sKV = s0 + 2 * C::QBUFS * C::TILE_BYTES;
  const uint32_t bars = s0 + C::DATA_BYTES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::DATA_BYTES + C::NUM_BARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* drain_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);  // stays 0
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 3);   // [2], per tile

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int G = gridDim.x;
  const int cta = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(bars + 8 * (C::B_Q_FULL + b), 1);
      mbar_init(bars + 8 * (C::B_Q_EMPTY + b), 1);
    }
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bars + 8 * (C::B_KV_FULL + s), 1);
      mbar_init(bars + 8 * (C::B_KV_EMPTY + s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bars + 8 * (C::B_S_FULL + i), 1);
      mbar_init(bars + 8 * (C::B_P_FULL + i), BM);
      mbar_init(bars + 8 * (C::B_P_HALF + i), BM);
      mbar_init(bars + 8 * (C::B_O_FULL + i), 1);
      mbar_init(bars + 8 * (C::B_PV_DONE + i), 1);
      mbar_init(bars + 8 * (C::B_WG + i), BM);
      last_flag[i] = 0;
    }
    mbar_init(bars + 8 * C::B_DRAIN, 1);
    *abort_flag = 0;
    *drain_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const unsigned long long tmo = p.timeout_ns;
  // Everything above touches no global memory; from here on the previous
  // kernel on the stream (which may have written q, k, v, o or the
  // workspace) must be complete. The next kernel may then be launched: its
  // CTAs take SMs only as this grid's CTAs exit.
  griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();

  if (warp >= 8) setmaxnreg_dec<REGS_CONTROL>();  // whole control warpgroup, one instruction
  if (warp == PRODUCER_WARP) {
    // ------------------------------------------------------------ producer
    // Whole-warp loop; one elected lane issues each TMA and expect-tx.
    {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      SegIter si;
      si.init(p, cta, G);
      int unit, t0, t1;
      bool fs;
      int it = 0, qseg = 0, q_issued = 0;
      bool ok = true;
      while (ok && si.next(unit, t0, t1, fs)) {
        const int bh = unit / p.n_qb;
        const int q_row0 = (unit - bh * p.n_qb) * p.unit_rows;
        const bool has1 = p.unit_rows == 2 * BM && (q_row0 + BM) < p.Sq;
        // Q buffer qb is free once every S MMA of the segment that last used
        // it (QBUFS segments ago) is done.
        const int qb = qseg % C::QBUFS;
        const uint32_t qfull = bars + 8 * (C::B_Q_FULL + qb);
        if (!bwait_warp(bars, C::B_Q_EMPTY + qb, ((qseg / C::QBUFS) & 1) ^ 1u, abort_flag, tmo, ROLE_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx_warp(qfull, (has1 ? 2 : 1) * C::TILE_BYTES);
#pragma unroll
        for (int c = 0; c < C::NCHUNK; ++c) {
          tma_load_3d_warp(sQ + (2 * qb) * C::TILE_BYTES + c * CHUNK_BYTES, &tm_q, qfull, c * 64, q_row0, bh);
          if (has1)
            tma_load_3d_warp(sQ + (2 * qb + 1) * C::TILE_BYTES + c * CHUNK_BYTES, &tm_q, qfull, c * 64,
                             q_row0 + BM, bh);
        }
        ++qseg;
        q_issued = 1;
        for (int j = t0; j < t1 && ok; ++j) {
          // one ring stage holds K(j) then V(j), under one barrier
          const int ps = it % C::PAIRS;
          const uint32_t ph = (it / C::PAIRS) & 1;
          if (!bwait_warp(bars, C::B_KV_EMPTY + ps, ph ^ 1u, abort_flag, tmo, ROLE_PRODUCER)) {
            ok = false;
            break;
          }
          const uint32_t full = bars + 8 * (C::B_KV_FULL + ps);
          mbar_arrive_expect_tx_warp(full, 2 * C::TILE_BYTES);
#pragma unroll
          for (int kv = 0; kv < 2; ++kv) {
            const CUtensorMap* m = kv ? &tm_v : &tm_k;
#pragma unroll
            for (int c = 0; c < C::NCHUNK; ++c)
              tma_load_3d_warp(sKV + (2 * ps + kv) * C::TILE_BYTES + c * CHUNK_BYTES, m, full, c * 64, j * BN, bh);
          }
          ++it;
        }
      }
      if (!ok) {
        // Drain: every load issued must land before the CTA's shared memory goes away.
        // the last Q load into each buffer
        for (int k = (qseg > C::QBUFS ? qseg - C::QBUFS : 0); q_issued && k < qseg; ++k) {
          const uint32_t qf = bars + 8 * (C::B_Q_FULL + k % C::QBUFS);
          if (!mbar_try_wait(qf, (k / C::QBUFS) & 1))
            wait_slow(qf, (k / C::QBUFS) & 1, drain_flag, 100000000ull, C::B_Q_FULL + k % C::QBUFS,
                      ROLE_PRODUCER);
        }
        const int first = it > C::PAIRS ? it - C::PAIRS : 0;
        for (int t = first; t < it; ++t) {
          const int slot = t % C::PAIRS;
          const uint32_t ph = (t / C::PAIRS) & 1;
          if (!mbar_try_wait(bars + 8 * (C::B_KV_FULL + slot), ph))
            wait_slow(bars + 8 * (C::B_KV_FULL + slot), ph, drain_flag, 100000000ull, C::B_KV_FULL + slot,
                      ROLE_PRODUCER);
        }
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // ----------------------------------------------------------- MMA issuer
    // The whole warp runs the issue loop with identical values (so descriptors
    // stay in uniform registers); elect.sync picks the lane that issues each
    // tcgen05.mma / tcgen05.commit.
    {
      constexpr uint32_t IDESC_QK = idesc_f16_f32(BM, BN, 0, 0);
      const int dpv = (p.D + 15) & ~15;  // PV N dimension (multiple of 16)
      const uint32_t idesc_pv = idesc_f16_f32(BM, dpv, 0, 1);
      const int ksteps = (p.D + 15) / 16;  // QK reduction steps over the head dim
      const uint32_t tS0 = tmem + 0, tS1 = tmem + 128;
      const uint32_t tO0 = tmem + 256, tO1 = tmem + 256 + DP;
      const uint32_t tP0 = tmem + C::P_COL, tP1 = tmem + C::P_COL + 64;  // own P columns (SEP_P)
      // Descriptors are built once; an MMA step only adds its byte offset >> 4
      // to the start-address field (all tiles lie below 256 KiB of shared
      // memory, so the field never carries into the next one).
      const uint64_t dQ = sdesc_sw128(sQ, 16, 1024);
      const uint64_t dK = sdesc_sw128(sKV, 16, 1024);            // K-major K tiles
      const uint64_t dV = sdesc_sw128(sKV, CHUNK_BYTES, 1024);   // MN-major V tiles
      // k-steps of 16 head dims: 32 bytes apart inside a 64-column chunk, chunks
      // CHUNK_BYTES apart; issued four at a time (one chunk per group).
      auto issue_qk = [&](uint32_t d_tmem, uint64_t dq, uint32_t kv_off) {
        const uint64_t kb = dK + (kv_off >> 4);
        if (DP == 128 || ksteps == 4) {
#pragma unroll
          for (int c = 0; c < DP / 64; ++c) {
            const uint32_t o = static_cast<uint32_t>(c * CHUNK_BYTES) >> 4;
            mma4_ss_warp(d_tmem, dq + o, dq + o + 2, dq + o + 4, dq + o + 6, kb + o, kb + o + 2, kb + o + 4,
                         kb + o + 6, IDESC_QK, c > 0 ? 1u : 0u);
          }
        } else {  // head dim below 64: only the k-steps that hold data
#pragma unroll
          for (int k = 0; k < DP / 16; ++k) {
            const uint32_t off = static_cast<uint32_t>((k >> 2) * CHUNK_BYTES + (k & 3) * 32) >> 4;
            if (k < ksteps) mma_f16_ss_warp(d_tmem, dq + off, kb + off, IDESC_QK, k > 0 ? 1u : 0u);
          }
        }
      };
      // PV in two halves: keys 0-63 once the first half of P is stored
      // (P_HALF), keys 64-127 once all of it is (P_FULL). Each barrier
      // completes once per tile, so a parity never falls two phases behind.
      auto issue_pv = [&](uint32_t d_tmem, uint32_t p_tmem, uint32_t v_off, bool acc, int ptile,
                          uint32_t par) -> bool {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          if (!bwait_warp(bars, (hh ? C::B_P_FULL : C::B_P_HALF) + ptile, par, abort_flag, tmo, ROLE_MMA))
            return false;
          tc_fence_after();
          // keys 64 hh .. 64 hh + 63: P columns 32 hh .., V rows 2048 bytes per 16 keys
          const uint64_t vb = dV + ((v_off + 4 * hh * 2048) >> 4);
          mma4_ts_warp(d_tmem, p_tmem + 32 * hh, vb, vb + 128, vb + 256, vb + 384, idesc_pv,
                       (acc || hh > 0) ? 1u : 0u);
        }
        return true;
      };
      // One half of PV (SEP_P order): keys 64 hh .. 64 hh + 63 once that half
      // of P is stored.
      auto pv_half = [&](uint32_t d_tmem, uint32_t p_tmem, uint32_t v_off, bool acc, int ptile, int hh,
                         uint32_t par) -> bool {
        if (!bwait_warp(bars, (hh ? C::B_P_FULL : C::B_P_HALF) + ptile, par, abort_flag, tmo, ROLE_MMA))
          return false;
        tc_fence_after();
        const uint64_t vb = dV + ((v_off + 4 * hh * 2048) >> 4);
        mma4_ts_warp(d_tmem, p_tmem + 32 * hh, vb, vb + 128, vb + 256, vb + 384, idesc_pv,
                     (acc || hh > 0) ? 1u : 0u);
        return true;
      };

      SegIter si;
      si.init(p, cta, G);
      int unit, t0, t1;
      bool fs;
      int it = 0, qseg = 0;
      uint32_t g0 = 0, g1 = 0;  // S/P phases completed per query tile
      bool ok = true;
      while (ok && si.next(unit, t0, t1, fs)) {
        const int bh = unit / p.n_qb;
        const int q_row0 = (unit - bh * p.n_qb) * p.unit_rows;
        const bool has1 = p.unit_rows == 2 * BM && (q_row0 + BM) < p.Sq;
        const int qb = qseg % C::QBUFS;
        if (!bwait_warp(bars, C::B_Q_FULL + qb, (qseg / C::QBUFS) & 1, abort_flag, tmo, ROLE_MMA)) { ok = false; break; }
        ++qseg;
        const uint64_t dQ0 = dQ + ((2 * qb) * C::TILE_BYTES >> 4);
        const uint64_t dQ1 = dQ + ((2 * qb + 1) * C::TILE_BYTES >> 4);
        tc_fence_after();
        if constexpr (C::SEP_P) {
          // S(j+1) of a query tile goes in right after the first half of PV(j):
          // the first-half P barrier also means the softmax has read all of
          // S(j) into registers, and P(j) has columns of its own. Per key
          // tile: PV0(j) keys 0-63, S0(j+1), PV0(j) keys 64-127, then the same
          // for query tile 1, then K(j) and V(j) are released.
          int ps = it % C::PAIRS;
          if (!bwait_warp(bars, C::B_KV_FULL + ps, (it / C::PAIRS) & 1, abort_flag, tmo, ROLE_MMA)) {
            ok = false;
            break;
          }
          ++it;
          tc_fence_after();
          issue_qk(tS0, dQ0, 2 * ps * C::TILE_BYTES);
          tc_commit_warp(bars + 8 * (C::B_S_FULL + 0));
          if (has1) {
            issue_qk(tS1, dQ1, 2 * ps * C::TILE_BYTES);
            tc_commit_warp(bars + 8 * (C::B_S_FULL + 1));
          }
          if (t1 - t0 == 1) tc_commit_warp(bars + 8 * (C::B_Q_EMPTY + qb));  // last S of the segment issued
          for (int j = t0; j < t1; ++j) {
            const bool nxt = j + 1 < t1;
            int nps = 0;
            if (nxt) {
              nps = it % C::PAIRS;
              if (!bwait_warp(bars, C::B_KV_FULL + nps, (it / C::PAIRS) & 1, abort_flag, tmo, ROLE_MMA)) {
                ok = false;
                break;
              }
              ++it;
              tc_fence_after();
            }
            const uint32_t v_off = (2 * ps + 1) * C::TILE_BYTES;
            if (!pv_half(tO0, tP0, v_off, j > t0, 0, 0, g0 & 1)) { ok = false; break; }
            if (nxt) {
              issue_qk(tS0, dQ0, 2 * nps * C::TILE_BYTES);
              tc_commit_warp(bars + 8 * (C::B_S_FULL + 0));
            }
            if (!pv_half(tO0, tP0, v_off, j > t0, 0, 1, g0 & 1)) { ok = false; break; }
            ++g0;
            tc_commit_warp(bars + 8 * ((nxt ? C::B_PV_DONE : C::B_O_FULL) + 0));
            if (has1) {
              if (!pv_half(tO1, tP1, v_off, j > t0, 1, 0, g1 & 1)) { ok = false; break; }
              if (nxt) {
                issue_qk(tS1, dQ1, 2 * nps * C::TILE_BYTES);
                tc_commit_warp(bars + 8 * (C::B_S_FULL + 1));
              }
              if (!pv_half(tO1, tP1, v_off, j > t0, 1, 1, g1 & 1)) { ok = false; break; }
              ++g1;
              tc_commit_warp(bars + 8 * ((nxt ? C::B_PV_DONE : C::B_O_FULL) + 1));
            }
            if (j + 2 == t1) tc_commit_warp(bars + 8 * (C::B_Q_EMPTY + qb));  // last S of the segment issued
            tc_commit_warp(bars + 8 * (C::B_KV_EMPTY + ps));  // K(j) and V(j) free
            ps = nps;
          }
          continue;
        }
        int prev_ps = 0;
        for (int j = t0; j < t1; ++j) {
          const int ps = it % C::PAIRS;
          const uint32_t kv_ph = (it / C::PAIRS) & 1;
          ++it;
          const int k_slot = 2 * ps, v_slot = 2 * ps + 1;
          const int prev_v_slot = 2 * prev_ps + 1;
          if (!bwait_warp(bars, C::B_KV_FULL + ps, kv_ph, abort_flag, tmo, ROLE_MMA)) { ok = false; break; }
          tc_fence_after();
          issue_qk(tS0, dQ0, k_slot * C::TILE_BYTES);  // S0(j); PV0(j-1) was issued before it
          tc_commit_warp(bars + 8 * (C::B_S_FULL + 0));
          if (has1) {
            if (j > t0) {
              if (!issue_pv(tO1, tS1, prev_v_slot * C::TILE_BYTES, j - 1 > t0, 1, (g1 - 1) & 1)) {
                ok = false;
                break;
              }
              tc_commit_warp(bars + 8 * (C::B_KV_EMPTY + prev_ps));  // K(j-1) and V(j-1) free
            }
            issue_qk(tS1, dQ1, k_slot * C::TILE_BYTES);
            tc_commit_warp(bars + 8 * (C::B_S_FULL + 1));
            ++g1;
          }
          if (j + 1 == t1) tc_commit_warp(bars + 8 * (C::B_Q_EMPTY + qb));  // last S of this segment issued
          // V(j) landed together with K(j) (one barrier per pair)
          if (!issue_pv(tO0, tS0, v_slot * C::TILE_BYTES, j > t0, 0, g0 & 1)) { ok = false; break; }
          ++g0;
          if (j + 1 == t1) tc_commit_warp(bars + 8 * (C::B_O_FULL + 0));  // tile 0 epilogue may start
          if (!has1) tc_commit_warp(bars + 8 * (C::B_KV_EMPTY + ps));
          prev_ps = ps;
        }
        if (ok && has1) {
          if (issue_pv(tO1, tS1, (2 * prev_ps + 1) * C::TILE_BYTES, t1 - 1 > t0, 1, (g1 - 1) & 1)) {
            tc_commit_warp(bars + 8 * (C::B_KV_EMPTY + prev_ps));
          } else {
            ok = false;
          }
        }
        if (ok && has1) tc_commit_warp(bars + 8 * (C::B_O_FULL + 1));
      }
      if (!ok) {
        // Drain every MMA issued so far before TMEM and shared memory are released.
        tc_commit_warp(bars + 8 * C::B_DRAIN);
        wait_slow(bars + 8 * C::B_DRAIN, 0, drain_flag, 100000000ull, C::B_DRAIN, ROLE_MMA);
      }
    }
    __syncwarp();
  } else if (warp < 8) {
    // ------------------------------------------------------------ softmax
    setmaxnreg_inc<REGS_SOFTMAX>();
    const int ti = warp >> 2;  // query tile
    const int quad = warp & 3; // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    const int role = ti ? ROLE_SOFTMAX1 : ROLE_SOFTMAX0;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off + ti * 128;
    const uint32_t tO = tmem + lane_off + 256 + ti * DP;
    // where P is stored: over S, or in its own columns (SEP_P)
    const uint32_t tP = C::SEP_P ? tmem + lane_off + C::P_COL + ti * 64 : tS;
    const float sl2 = p.scale_log2;
    const bool pos = sl2 >= 0.f;
    SegIter si;
    si.init(p, cta, G);
    int unit, t0, t1;
    bool first_seg;
    uint32_t g = 0, oseg = 0, wsync = 0, pvg = 0;
    bool ok = true;
    auto wg_sync = [&]() -> bool {
      mbar_arrive(bars + 8 * (C::B_WG + ti));
      const bool r = bwait_warp(bars, C::B_WG + ti, wsync & 1, abort_flag, tmo, role);
      ++wsync;
      return r;
    };
    while (ok && si.next(unit, t0, t1, first_seg)) {
      const int bh = unit / p.n_qb;
      const int q_row0 = (unit - bh * p.n_qb) * p.unit_rows;
      const bool has1 = p.unit_rows == 2 * BM && (q_row0 + BM) < p.Sq;
      if (ti == 1 && !has1) continue;
      float m_run = -INFINITY;  // running max, already multiplied by scale*log2(e)
      float l_run = 0.f;
      for (int j = t0; j < t1; ++j) {
        if (!bwait_warp(bars, C::B_S_FULL + ti, g & 1, abort_flag, tmo, role)) { ok = false; break; }
        tc_fence_after();
        uint32_t s[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS + 32 * c, s + 32 * c);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) reg_fence32(s + 32 * c);

        const int nvalid = min(BN, p.Skv - j * BN);
        const bool full = nvalid == BN;
        const float mx = row_extreme(s, nvalid, full, pos);
        const float m_cand = mx * sl2;
        const float m_new = fmaxf(m_run, m_cand);
        const bool need = m_new > m_run + RESCALE_THRESHOLD;
        float factor = 1.f;
        if (need) {
          factor = ex2_approx(m_run - m_new);  // 0 on the first tile (m_run = -inf)
          m_run = m_new;
        }
        // Rescale this warp's O rows when any of them moved its max, before any
        // of P is published; PV(j) waits for the P barriers. 16 columns at a
        // time: the whole score row is live here, and 32 more registers would
        // spill (measured on B200: the spill-free form is 4-7% faster at D=128).
        if constexpr (!C::SEP_P) rescale_rows<DP>(tO, j > t0 && __any_sync(0xffffffffu, need), factor);
        // Over S, PV(j-1) of this tile completed before S(j) was signalled.
        // With P in its own columns S(j) is computed while PV(j-1) may still
        // run: wait for PV(j-1) (it reads P and accumulates O) only before
        // the first P store, after the first half's exponentials.
        bool pv_ok = true;
        auto before_store = [&] {
          if constexpr (C::SEP_P) {
            if (j > t0) {
              pv_ok = bwait_warp(bars, C::B_PV_DONE + ti, pvg & 1, abort_flag, tmo, role);
              ++pvg;
              tc_fence_after();
              rescale_rows<DP>(tO, __any_sync(0xffffffffu, need), factor);
            }
          }
        };
        l_run *= factor;
        const float neg_m = -m_run;
        const uint32_t half_bar = bars + 8 * (C::B_P_HALF + ti);
        float lsum0, lsum1;
        if (full)
          row_exp_store<false>(s, sl2, neg_m, nvalid, tP, lsum0, lsum1, half_bar, [] {}, before_store);
        else
          row_exp_store<true>(s, sl2, neg_m, nvalid, tP, lsum0, lsum1, half_bar, [] {}, before_store);
        l_run += lsum0 + lsum1;
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bars + 8 * (C::B_P_FULL + ti));
        ++g;
        if (!pv_ok) { ok = false; break; }
      }
      if (!ok) break;
      // -------------------------------------------------- segment epilogue
      if (!bwait_warp(bars, C::B_O_FULL + ti, oseg & 1, abort_flag, tmo, role)) { ok = false; break; }
      ++oseg;
      tc_fence_after();
      // Output goes through this warp's staging tile at s0 + EPI_OFF + warp * 4 KiB
      // (rows q_row0 + ti * BM + quad * 32 + 0..31). The addresses are formed
      // where they are used: kept in registers across the branch they made the
      // compiler spill at D = 128.
      if (t0 == 0 && t1 == p.n_tiles) {
        // whole unit: O / l to global memory through the staging tile
        const float inv = 1.f / l_run;
#pragma unroll
        for (int hf = 0; hf < DP / 64; ++hf) {
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            uint32_t o[32];
            tmem_ld32(tO + 64 * hf + 32 * cc, o);
            tmem_wait_ld();
            reg_fence32(o);
            stage_32(s0 + C::EPI_OFF + warp * 4096, lane, cc, o, inv);
          }
          flush_stage(s0 + C::EPI_OFF + warp * 4096, lane, p.o + static_cast<long long>(bh) * p.Sq * p.D,
                      q_row0 + ti * BM + quad * 32, p.Sq, p.D, 64 * hf);
        }
        continue;
      }
      // partial piece: unnormalised O, m and l to this CTA's workspace slot
      const int which = first_seg ? 0 : 1;
      const long long slot = (static_cast<long long>(cta) * 2 + which) * 2 + ti;
      // chunk-major slot: 4 columns of one row are 16 bytes, the 128 rows of a
      // 4-column chunk are contiguous, so a warp's 32 rows store 512
      // contiguous bytes per instruction (row-major, every store touched 32 lines)
      float* wo = p.ws_o + slot * BM * DP + row * 4;
      float* wml = p.ws_ml + (slot * BM + row) * 2;
#pragma unroll
      for (int c = 0; c < DP / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + 32 * c, o);
        tmem_wait_ld();
        reg_fence32(o);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          *reinterpret_cast<float4*>(wo + (c * 8 + e) * BM * 4) = make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]),
                               __uint_as_float(o[4 * e + 2]), __uint_as_float(o[4 * e + 3]));
      }
      *reinterpret_cast<float2*>(wml) = make_float2(m_run, l_run);
      // Units of few pieces are combined here by the piece that finishes
      // last, overlapping the other CTAs' work; units of many pieces by
      // attn_combine_kernel, launched after this grid (p.combine == 0).
      if (!p.combine) continue;
      // Release: the warpgroup rendezvous orders every thread's stores before
      // thread 0's gpu-scope fence, which orders them before the counter.
      if (!wg_sync()) { ok = false; break; }
      const int rel = unit - p.tail_unit0;  // index of the unit within the split tail
      unsigned long long* cnt = p.ws_cnt + rel * 2 + ti;
      const long long W = p.total_steps;
      const int GT = p.tail_ctas;
      const long long ubase = static_cast<long long>(rel) * p.n_tiles;
      const int c_lo = owner_cta(ubase, W, GT);
      const int c_hi = owner_cta(ubase + p.n_tiles - 1, W, GT);
      if (quad == 0 && lane == 0) {
        __threadfence();
        // A counter whose tag is not this launch's epoch counts as 0, so the
        // workspace needs no clearing between calls of any size.
        unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(cnt), next;
        while (true) {
          next = (((cur >> 8) == p.epoch) ? cur : (p.epoch << 8)) + 1ull;
          const unsigned long long seen = atomicCAS(cnt, cur, next);
          if (seen == cur) break;
          cur = seen;
        }
        const int last = (static_cast<int>(next & 0xffull) == c_hi - c_lo + 1) ? 1 : 0;
        if (last) __threadfence();  // acquire: the other pieces' stores are visible
        last_flag[ti] = last;
      }
      if (!wg_sync()) { ok = false; break; }
      if (last_flag[ti]) {
        // Last piece to finish: combine every piece of this (unit, query tile)
        // from the workspace, in CTA order whoever combines (deterministic
        // bits). One row per thread, all 128 rows in flight. A unit spans up
        // to MAX_PIECES CTA ranges, so the pieces are walked in a loop; each
        // piece's (m, l) pair is re-read (8 bytes, from L1/L2) where it is
        // needed instead of being held in registers for every piece.
        const int np = c_hi - c_lo + 1;  // <= MAX_PIECES (make_plan guarantees it)
        // element offset of this row in piece k's slot: range c_lo + k starts
        // inside this unit (its first tail segment) iff floor(c * W / GT) >=
        // ubase, i.e. c * W >= ubase * GT
        auto piece_row = [&](int k) -> long long {
          const int c2 = c_lo + k;
          const int which2 = (static_cast<long long>(c2) * W >= ubase * GT) ? 0 : 1;
          return ((static_cast<long long>(c2) * 2 + which2) * 2 + ti) * BM + row;  // (slot, row)
        };
        auto piece_ml = [&](long long rb) -> float2 {
          return __ldcg(reinterpret_cast<const float2*>(p.ws_ml + rb * 2));
        };
        float m_all = -INFINITY;
#pragma unroll 1
        for (int k = 0; k < np; ++k) m_all = fmaxf(m_all, piece_ml(piece_row(k)).x);
        float l_all = 0.f;
#pragma unroll 1
        for (int k = 0; k < np; ++k) {
          const float2 ml = piece_ml(piece_row(k));
          l_all = fmaf(ml.y, ex2_approx(ml.x - m_all), l_all);
        }
        const float inv = 1.f / l_all;
#pragma unroll 1
        for (int c = 0; c < DP / 32; ++c) {
          float acc[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[e] = 0.f;
          // pieces two at a time: the loads of both are in flight together
          // (L2 latency, not bandwidth, bounds this loop); the accumulation
          // order is still piece 0, 1, 2, ...
#pragma unroll 1
          for (int k0 = 0; k0 < np; k0 += 2) {
            float4 v4[2][8];
            float wk[2];
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const int k = (k0 + kk < np) ? k0 + kk : k0;  // a duplicate load, never accumulated
              const long long rb = piece_row(k);
              wk[kk] = ex2_approx(piece_ml(rb).x - m_all);
              // chunk-major slot (see the partial write): chunk q of this row
              const long long sl = rb / BM;
              const float* sbase = p.ws_o + sl * BM * DP + (rb - sl * BM) * 4;
#pragma unroll
              for (int e = 0; e < 8; ++e)
                v4[kk][e] = __ldcg(reinterpret_cast<const float4*>(sbase + (c * 8 + e) * BM * 4));
            }
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              if (k0 + kk < np) {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  acc[4 * e] = fmaf(v4[kk][e].x, wk[kk], acc[4 * e]);
                  acc[4 * e + 1] = fmaf(v4[kk][e].y, wk[kk], acc[4 * e + 1]);
                  acc[4 * e + 2] = fmaf(v4[kk][e].z, wk[kk], acc[4 * e + 2]);
                  acc[4 * e + 3] = fmaf(v4[kk][e].w, wk[kk], acc[4 * e + 3]);
                }
              }
            }
          }
          uint32_t o[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(acc[e]);
          stage_32(s0 + C::EPI_OFF + warp * 4096, lane, c & 1, o, inv);
          if (c & 1)
            flush_stage(s0 + C::EPI_OFF + warp * 4096, lane, p.o + static_cast<long long>(bh) * p.Sq * p.D,
                        q_row0 + ti * BM + quad * 32, p.Sq, p.D, 64 * (c >> 1));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------- D = 512 on CTA pairs
// Head dim 512 (the reference's VAE mid-block path, attn_kernel.hip:525-708).
// An fp32 O tile of 128 rows x 512 columns fills all of TMEM, so O is split
// into two 256-column halves of the head dim, and both halves compute the
// full S = Q K^T (K = 512): 1.5x the minimum tensor work, in exchange for no
// traffic between the halves. TMEM per CTA: S double-buffered at [0,128) /
// [128,256), the O half at [256,512); P of a key tile is written over the
// first 64 columns of its S buffer; MMA order S(0), S(1), PV(0), S(2),
// PV(1), ... so that the tensor core computes S(j+1) while the softmax works
// on S(j).
//
// Work runs on 2-CTA clusters: a work unit is two query tiles of one (batch,
// head) and one head-dim half, one query tile per CTA. The even CTA (the
// leader) issues every MMA with
// cta_group::2: M = 256 rows, 128 from each CTA's Q tile, D in each CTA's own
// TMEM. Each CTA loads only half of the B operands into its shared memory:
// keys 64 r .. 64 r + 63 of every K tile and head dims 128 r .. 128 r + 127
// of its half of every V tile (r = CTA rank), so a CTA streams 96 KiB per key
// tile instead of 192 KiB and its three 32 KiB ring slots each feed 1024
// tensor cycles instead of 512 (measured on B200: with one CTA per (query
// tile, half) the MMA warp waited 19% of the time for K/V data; here 11%).
//
// Persistent: one cluster per SM pair walks a list of segments (unit, first
// key tile, end key tile) with the schedule of attn_fwd_kernel (SegIter over
// clusters): whole units first, then, in split mode, the key range of the
// last partial wave cut into contiguous step ranges per cluster, partial
// results combined by the last piece to finish (one combine per unit and
// CTA rank). Without it 256 one-shot CTAs (C4) made 1.73 waves on 148 SMs.
//
// Ring slots per key tile j (both CTAs, the same sequence): K(j) head dims
// 0-255, K(j) head dims 256-511, then V(j-1). A slot of K is four 8 KiB
// [64 keys x 64 dims] boxes; a slot of V two 16 KiB [128 keys x 64 dims] boxes.
//
// Protocol (per slot phase): each producer waits for its own KV_EMPTY (the
// leader's MMA commit arrives in both CTAs), the leader's producer arms the
// leader's KV_FULL for the bytes of both CTAs, and both CTAs' loads complete on
// the leader's KV_FULL; Q the same way per segment, after this CTA's Q_EMPTY
// (its previous segment's epilogue has released the Q buffer, which stages a
// whole unit's output for its TMA store). The leader's MMA warp waits on
// KV_FULL and on P_FULL, which both softmax warpgroups arrive at (the odd
// CTA's remotely); S_FULL, PV_DONE and O_FULL are multicast commits that
// arrive in both CTAs.
struct Cfg512P {
  static constexpr int SLOTS = 3;
  static constexpr int SLOT_BYTES = 2 * CHUNK_BYTES;
  static constexpr int Q_BYTES = 8 * CHUNK_BYTES;
  static constexpr int DATA_BYTES = Q_BYTES + SLOTS * SLOT_BYTES;
  static constexpr int B_Q = 0, B_Q_EMPTY = 1, B_KV_FULL = 2, B_KV_EMPTY = 2 + SLOTS, B_S_FULL = 2 + 2 * SLOTS;
  static constexpr int B_P_FULL = B_S_FULL + 2, B_PV_DONE = B_P_FULL + 2, B_O_FULL = B_PV_DONE + 1;
  static constexpr int B_DRAIN = B_O_FULL + 1, B_EPI = B_DRAIN + 1, NUM_BARS = B_EPI + 1;
  static constexpr int SMEM_BYTES = 1024 + DATA_BYTES + NUM_BARS * 8 + 16;
  static constexpr int THREADS = 256;
  static constexpr int DH = 256;  // head dims per CTA pair (one half of D = 512)
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ bool bwait_cluster_warp(uint32_t bars, int idx, uint32_t parity, volatile int* abort_flag,
                                                   unsigned long long timeout_ns, int role) {
  const uint32_t bar = bars + 8u * idx;
  bool ok = mbar_try_wait_cluster(bar, parity);
  if (!ok) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t n = 0;
    while (true) {
      if (mbar_try_wait_cluster(bar, parity)) { ok = true; break; }
      if (*abort_flag) break;
      if ((++n & 31u) == 0u) {
        const uint64_t t = globaltimer_ns();
        if (t - t0 > timeout_ns || n > (1u << 24)) {
          *abort_flag = 1;
          if (atomicCAS(&g_status, 0u, 1u) == 0u) {
            g_timeout_info[0] = blockIdx.x;
            g_timeout_info[1] = blockIdx.y;
            g_timeout_info[2] = threadIdx.x / 32;
            g_timeout_info[3] = idx;
            g_timeout_info[4] = static_cast<int>(parity);
            g_timeout_info[5] = role;
            __threadfence();
          } else {
            atomicOr(&g_status, 1u);
          }
          break;
        }
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

// Unit u of the D = 512 pair schedule: p.n_qb units per (batch, head), each
// (query tile pair, head-dim half); this CTA's query rows and head-dim half.
struct Unit512 {
  int bh, half, q_row0;
  __device__ __forceinline__ Unit512(const Params& p, int u, uint32_t rank) {
    bh = u / p.n_qb;
    const int rem = u - bh * p.n_qb;
    half = rem & 1;
    q_row0 = ((rem >> 1) * 2 + static_cast<int>(rank)) * BM;
  }
};

// DMAJOR: q, k, v and o are stored transposed, [B*H][D][S] with the sequence
// contiguous -- a [b, c, h, w] feature map is exactly this with H = 1, D = c,
// S = h*w -- and the kernel reads and writes that layout directly: Q and K
// become MN-major MMA operands (64 sequence positions per 128-byte row, head
// dims down the rows), V a K-major one, and O is staged as [256 d][128 rows]
// and written with one unswizzled TMA store. Whole units only (no workspace).
template <bool DMAJOR>
__global__ void __launch_bounds__(Cfg512P::THREADS, 1)
    attn_fwd_d512_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                              const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                              const Params p) {
  using C = Cfg512P;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t s0 = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (s0 - raw);
  const uint32_t sQ = s0;
  const uint32_t sRing = s0 + C::Q_BYTES;
  const uint32_t bars = s0 + C::DATA_BYTES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::DATA_BYTES + C::NUM_BARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* drain_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();  // 0: leader (issues the MMAs), 1: peer
  const bool leader = rank == 0;
  const int cl = blockIdx.x >> 1;   // cluster index
  const int Gc = gridDim.x >> 1;    // clusters
  const unsigned long long tmo = p.timeout_ns;

  if (threadIdx.x == 0) {
    mbar_init(bars + 8 * C::B_Q, 1);
    mbar_init(bars + 8 * C::B_Q_EMPTY, 1);
    for (int s = 0; s < C::SLOTS; ++s) {
      mbar_init(bars + 8 * (C::B_KV_FULL + s), 1);
      mbar_init(bars + 8 * (C::B_KV_EMPTY + s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bars + 8 * (C::B_S_FULL + i), 1);
      mbar_init(bars + 8 * (C::B_P_FULL + i), 2 * BM);  // both CTAs' softmax threads (leader's barrier)
    }
    mbar_init(bars + 8 * C::B_PV_DONE, 1);
    mbar_init(bars + 8 * C::B_O_FULL, 1);
    mbar_init(bars + 8 * C::B_DRAIN, 1);
    mbar_init(bars + 8 * C::B_EPI, BM);
    *abort_flag = 0;
    *drain_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 5) {
    tmem_alloc2(smem_u32(tmem_slot), 512);
    tmem_relinquish2();
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_o);
    const uint32_t lead_q = mapa_shared(bars + 8 * C::B_Q, 0);
    SegIter si;
    si.init(p, cl, Gc);
    int unit, t0, t1;
    bool fs;
    int it = 0, qseg = 0;
    bool ok = true;
    auto slot_begin = [&](int& slot, uint32_t& lead_full) -> bool {
      slot = it % C::SLOTS;
      const uint32_t ph = (it / C::SLOTS) & 1;
      if (!bwait_warp(bars, C::B_KV_EMPTY + slot, ph ^ 1u, abort_flag, tmo, ROLE_PRODUCER)) return false;
      if (leader) mbar_arrive_expect_tx_warp(bars + 8 * (C::B_KV_FULL + slot), 2 * C::SLOT_BYTES);
      lead_full = mapa_shared(bars + 8 * (C::B_KV_FULL + slot), 0);
      ++it;
      return true;
    };
    while (ok && si.next(unit, t0, t1, fs)) {
      const Unit512 u(p, unit, rank);
      // the Q buffer is free once this CTA's previous segment is finished with it
      if (!bwait_warp(bars, C::B_Q_EMPTY, (qseg & 1) ^ 1u, abort_flag, tmo, ROLE_PRODUCER)) { ok = false; break; }
      if (leader) mbar_arrive_expect_tx_warp(bars + 8 * C::B_Q, 2 * C::Q_BYTES);
      if (DMAJOR) {
        // [64 rows x 256 dims] boxes: 64-row M block mb at 64 KiB * mb, one 128-byte row per head dim
        for (int mb = 0; mb < 2; ++mb)
          for (int dd = 0; dd < 2; ++dd)
            tma_load_3d_pair_warp(sQ + mb * 65536 + dd * 32768, &tm_q, lead_q, u.q_row0 + 64 * mb, 256 * dd, u.bh);
      } else {
        for (int c = 0; c < 8; ++c) tma_load_3d_pair_warp(sQ + c * CHUNK_BYTES, &tm_q, lead_q, c * 64, u.q_row0, u.bh);
      }
      ++qseg;
      for (int j = t0; j <= t1 && ok; ++j) {
        if (j < t1) {
          // K(j): keys j*128 + 64*rank .. +63, head dims 256 s .. 256 s + 255
          for (int s = 0; s < 2 && ok; ++s) {
            int slot;
            uint32_t lf;
            if (!(ok = slot_begin(slot, lf))) break;
            if (DMAJOR) {  // one [64 keys x 256 dims] box: a 128-byte row per head dim
              tma_load_3d_pair_warp(sRing + slot * C::SLOT_BYTES, &tm_k, lf, j * BN + 64 * static_cast<int>(rank),
                                    256 * s, u.bh);
            } else {
#pragma unroll
              for (int b = 0; b < 4; ++b)
                tma_load_3d_pair_warp(sRing + slot * C::SLOT_BYTES + b * 8192, &tm_k, lf, 256 * s + 64 * b,
                                      j * BN + 64 * static_cast<int>(rank), u.bh);
            }
          }
        }
        if (j > t0 && ok) {
          // V(j-1): keys (j-1)*128 .. +127, head dims 256 half + 128 rank .. +127
          int slot;
          uint32_t lf;
          if (!(ok = slot_begin(slot, lf))) break;
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            if (DMAJOR)  // [64 keys x 128 dims] boxes: keys 0-63, then 64-127
              tma_load_3d_pair_warp(sRing + slot * C::SLOT_BYTES + b * CHUNK_BYTES, &tm_v, lf, (j - 1) * BN + 64 * b,
                                    C::DH * u.half + 128 * static_cast<int>(rank), u.bh);
            else         // [128 keys x 64 dims] boxes
              tma_load_3d_pair_warp(sRing + slot * C::SLOT_BYTES + b * CHUNK_BYTES, &tm_v, lf,
                                    C::DH * u.half + 128 * static_cast<int>(rank) + 64 * b, (j - 1) * BN, u.bh);
          }
        }
      }
    }
    if (!ok && leader) {
      // Drain: every load issued must land before shared memory goes away.
      if (qseg > 0 && !mbar_try_wait(bars + 8 * C::B_Q, (qseg - 1) & 1))
        wait_slow(bars + 8 * C::B_Q, (qseg - 1) & 1, drain_flag, 100000000ull, C::B_Q, ROLE_PRODUCER);
      const int first = it > C::SLOTS ? it - C::SLOTS : 0;
      for (int t = first; t < it; ++t) {
        const int slot = t % C::SLOTS;
        const uint32_t ph = (t / C::SLOTS) & 1;
        if (!mbar_try_wait(bars + 8 * (C::B_KV_FULL + slot), ph))
          wait_slow(bars + 8 * (C::B_KV_FULL + slot), ph, drain_flag, 100000000ull, C::B_KV_FULL + slot,
                    ROLE_PRODUCER);
      }
    }
    __syncwarp();
  } else if (warp == 5 && leader) {
    // ----------------------------------------------------------- MMA issuer
    // Row-major: Q and K K-major, V MN-major. DMAJOR: Q and K MN-major (Q's
    // second 64-row M block 64 KiB on; a CTA's 64 keys are one N block), V
    // K-major (keys 64-127 one 16 KiB box on).
    constexpr uint32_t IDESC_QK = idesc_f16_f32(2 * BM, BN, DMAJOR ? 1 : 0, DMAJOR ? 1 : 0);  // M = 256, N = 128 keys
    constexpr uint32_t IDESC_PV = idesc_f16_f32(2 * BM, C::DH, 0, DMAJOR ? 0 : 1);  // N = 256 head dims of this half
    const uint64_t dQ = sdesc_sw128(sQ, DMAJOR ? 65536 : 16, 1024);
    const uint64_t dK = sdesc_sw128(sRing, DMAJOR ? 8192 : 16, 1024);
    const uint64_t dV = sdesc_sw128(sRing, DMAJOR ? 16 : CHUNK_BYTES, 1024);
    // descriptor steps of 16 head dims (S) / 16 keys (PV), in 16-byte units
    constexpr uint32_t QK_STEP = DMAJOR ? 128u : 2u;  // 16 rows of 128 B, or 32 B inside a row
    constexpr uint32_t PV_STEP = DMAJOR ? 2u : 128u;
    const uint32_t tO = tmem + 256;
    constexpr uint16_t BOTH = 0x3;
    int it = 0, qseg = 0;
    uint32_t gs = 0;  // S tiles issued (S / P buffer and phase)
    auto next_slot = [&](int& slot) -> bool {
      slot = it % C::SLOTS;
      const uint32_t ph = (it / C::SLOTS) & 1;
      ++it;
      if (!bwait_warp(bars, C::B_KV_FULL + slot, ph, abort_flag, tmo, ROLE_MMA)) return false;
      tc_fence_after();
      return true;
    };
    auto issue_s = [&](uint32_t g) -> bool {
      const uint32_t tS = tmem + 128 * (g & 1);
      for (int s = 0; s < 2; ++s) {
        int slot;
        if (!next_slot(slot)) return false;
        const uint32_t soff = static_cast<uint32_t>(slot * C::SLOT_BYTES) >> 4;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          // head dims 256 s + 64 b ..: row-major, Q chunk 4 s + b and K box b
          // (16 dims = 32 bytes); DMAJOR, 128-byte rows 256 s + 64 b .. of Q
          // and 64 b .. of the K slot (both 8 KiB per 64 dims)
          const uint64_t qa = dQ + (DMAJOR ? static_cast<uint32_t>((256 * s + 64 * b) * 128) >> 4
                                           : static_cast<uint32_t>((4 * s + b) * CHUNK_BYTES) >> 4);
          const uint64_t kb = dK + soff + (static_cast<uint32_t>(b * 8192) >> 4);
          mma4_ss_pair_warp(tS, qa, qa + QK_STEP, qa + 2 * QK_STEP, qa + 3 * QK_STEP, kb, kb + QK_STEP,
                            kb + 2 * QK_STEP, kb + 3 * QK_STEP, IDESC_QK, (s > 0 || b > 0) ? 1u : 0u);
        }
        tc_commit_pair_mc_warp(bars + 8 * (C::B_KV_EMPTY + slot), BOTH);
      }
      tc_commit_pair_mc_warp(bars + 8 * (C::B_S_FULL + (g & 1)), BOTH);
      return true;
    };
    // PV of S tile g; acc: accumulate into O (not the segment's first key tile);
    // last: the segment's last key tile (O_FULL instead of PV_DONE)
    auto issue_pv = [&](uint32_t g, bool acc, bool last) -> bool {
      if (!bwait_cluster_warp(bars, C::B_P_FULL + (g & 1), (g >> 1) & 1, abort_flag, tmo, ROLE_MMA)) return false;
      tc_fence_after();
      const uint32_t tP = tmem + 128 * (g & 1);
      int slot;
      if (!next_slot(slot)) return false;
      const uint32_t soff = static_cast<uint32_t>(slot * C::SLOT_BYTES) >> 4;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        // keys 64 c .. 64 c + 63: P columns 32 c ..; row-major, V rows 2048
        // bytes per 16 keys; DMAJOR, the second 16 KiB box, 32 bytes per 16 keys
        const uint64_t vb = dV + soff + (static_cast<uint32_t>(DMAJOR ? c * CHUNK_BYTES : 4 * c * 2048) >> 4);
        mma4_ts_pair_warp(tO, tP + 32 * c, vb, vb + PV_STEP, vb + 2 * PV_STEP, vb + 3 * PV_STEP, IDESC_PV,
                          (acc || c > 0) ? 1u : 0u);
      }
      tc_commit_pair_mc_warp(bars + 8 * (C::B_KV_EMPTY + slot), BOTH);
      tc_commit_pair_mc_warp(bars + 8 * (last ? C::B_O_FULL : C::B_PV_DONE), BOTH);
      return true;
    };
    SegIter si;
    si.init(p, cl, Gc);
    int unit, t0, t1;
    bool fs;
    bool ok = true;
    while (ok && si.next(unit, t0, t1, fs)) {
      if (!bwait_warp(bars, C::B_Q, qseg & 1, abort_flag, tmo, ROLE_MMA)) { ok = false; break; }
      ++qseg;
      tc_fence_after();
      const uint32_t g0 = gs;
      for (int j = t0; j <= t1 && ok; ++j) {
        if (j < t1) ok = issue_s(gs++);
        if (ok && j > t0) ok = issue_pv(g0 + (j - 1 - t0), j - 1 > t0, j == t1);
      }
    }
    if (!ok) {
      tc_commit_pair_mc_warp(bars + 8 * C::B_DRAIN, 0x1);
      wait_slow(bars + 8 * C::B_DRAIN, 0, drain_flag, 100000000ull, C::B_DRAIN, ROLE_MMA);
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------------------- softmax
    const int row = warp * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tO = tmem + lane_off + 256;
    const float sl2 = p.scale_log2;
    const bool pos = sl2 >= 0.f;
    const uint32_t p_full0 = mapa_shared(bars + 8 * C::B_P_FULL, 0);  // the leader's P_FULL[0]
    SegIter si;
    si.init(p, cl, Gc);
    int unit, t0, t1;
    bool first_seg;
    uint32_t gs = 0, pvg = 0, oseg = 0, epi = 0;
    bool ok = true;
    while (ok && si.next(unit, t0, t1, first_seg)) {
      const Unit512 u(p, unit, rank);
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = t0; j < t1; ++j) {
        const int b = gs & 1;
        const uint32_t tS = tmem + lane_off + 128 * b;
        if (!bwait_warp(bars, C::B_S_FULL + b, (gs >> 1) & 1, abort_flag, tmo, ROLE_SOFTMAX0)) { ok = false; break; }
        tc_fence_after();
        uint32_t s[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS + 32 * c, s + 32 * c);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) reg_fence32(s + 32 * c);
        const int nvalid = min(BN, p.Skv - j * BN);
        const bool full = nvalid == BN;
        const float mx = row_extreme(s, nvalid, full, pos);
        const float m_new = fmaxf(m_run, mx * sl2);
        const bool need = m_new > m_run + RESCALE_THRESHOLD;
        float factor = 1.f;
        if (need) {
          factor = ex2_approx(m_run - m_new);
          m_run = m_new;
        }
        l_run *= factor;
        float lsum0, lsum1;
        if (full)
          row_exp_store<false>(s, sl2, -m_run, nvalid, tS, lsum0, lsum1, 0u, [] {}, [] {});
        else
          row_exp_store<true>(s, sl2, -m_run, nvalid, tS, lsum0, lsum1, 0u, [] {}, [] {});
        l_run += lsum0 + lsum1;
        // O may only be rescaled once PV(j-1) has completed.
        if (j > t0) {
          if (!bwait_warp(bars, C::B_PV_DONE, pvg & 1, abort_flag, tmo, ROLE_SOFTMAX0)) { ok = false; break; }
          ++pvg;
          tc_fence_after();
          if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
            for (int c = 0; c < C::DH / 32; ++c) {
              uint32_t o[32];
              tmem_ld32(tO + 32 * c, o);
              tmem_wait_ld();
              reg_fence32(o);
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
              tmem_st32(tO + 32 * c, o);
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive_remote(p_full0 + 8u * b);  // the leader's P_FULL[b]
        ++gs;
      }
      if (!ok) break;
      // -------------------------------------------------- segment epilogue
      if (!bwait_warp(bars, C::B_O_FULL, oseg & 1, abort_flag, tmo, ROLE_SOFTMAX0)) { ok = false; break; }
      ++oseg;
      tc_fence_after();
      if (t0 == 0 && t1 == p.n_tiles) {
        // whole unit: O / l staged in the Q buffer (its last MMA completed)
        // and written with TMA; then the buffer is released for the next Q
        const float inv = 1.f / l_run;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[64];
          tmem_ld32(tO + 64 * c, o);
          tmem_ld32(tO + 64 * c + 32, o + 32);
          tmem_wait_ld();
          reg_fence32(o);
          reg_fence32(o + 32);
          if (DMAJOR) {  // [256 dims][128 rows] fp16: this row is column `row`
#pragma unroll
            for (int e = 0; e < 64; ++e)
              st_shared_u16(sQ + ((64 * c + e) * BM + row) * 2,
                            __half_as_ushort(__float2half_rn(__uint_as_float(o[e]) * inv)));
            continue;
          }
          const uint32_t rowbase = sQ + c * CHUNK_BYTES + row * 128;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t a = pack_half2(__uint_as_float(o[8 * e + 0]) * inv, __uint_as_float(o[8 * e + 1]) * inv);
            const uint32_t bb = pack_half2(__uint_as_float(o[8 * e + 2]) * inv, __uint_as_float(o[8 * e + 3]) * inv);
            const uint32_t cc = pack_half2(__uint_as_float(o[8 * e + 4]) * inv, __uint_as_float(o[8 * e + 5]) * inv);
            const uint32_t d = pack_half2(__uint_as_float(o[8 * e + 6]) * inv, __uint_as_float(o[8 * e + 7]) * inv);
            st_shared_v4(rowbase + ((e ^ (row & 7)) << 4), a, bb, cc, d);
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(bars + 8 * C::B_EPI);
        const bool epi_ok = bwait_warp(bars, C::B_EPI, epi & 1, abort_flag, tmo, ROLE_SOFTMAX0);
        ++epi;
        if (!epi_ok) { ok = false; break; }
        if (warp == 0) {
          // (the odd CTA of the last pair may hold rows past Sq only: nothing to store)
          if (lane == 0 && u.q_row0 < p.Sq) {
            if (DMAJOR)  // one [128 rows x 256 dims] box
              tma_store_3d(&tm_o, sQ, u.q_row0, C::DH * u.half, u.bh);
            else
              for (int c = 0; c < 4; ++c)
                tma_store_3d(&tm_o, sQ + c * CHUNK_BYTES, C::DH * u.half + 64 * c, u.q_row0, u.bh);
            tma_store_commit();
            tma_store_wait_read0();
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(bars + 8 * C::B_Q_EMPTY);
        }
        continue;
      }
      // partial piece: the Q buffer is not needed for it
      if (warp == 0 && lane == 0) mbar_arrive(bars + 8 * C::B_Q_EMPTY);
      // unnormalised O, m and l of this CTA's rows to its workspace slot,
      // chunk-major: [DH/4][128 rows][4] fp32
      const int which = first_seg ? 0 : 1;
      const long long slot = (static_cast<long long>(cl) * 2 + rank) * 2 + which;
      float* wo = p.ws_o + slot * BM * C::DH + row * 4;
#pragma unroll 1
      for (int c = 0; c < C::DH / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + 32 * c, o);
        tmem_wait_ld();
        reg_fence32(o);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          *reinterpret_cast<float4*>(wo + (c * 8 + e) * BM * 4) =
              make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]), __uint_as_float(o[4 * e + 2]),
                          __uint_as_float(o[4 * e + 3]));
      }
      *reinterpret_cast<float2*>(p.ws_ml + (slot * BM + row) * 2) = make_float2(m_run, l_run);
      // attn_combine_kernel, launched after this grid, combines the pieces
    }
  }

  // Neither CTA may release its shared memory or TMEM while the other (or
  // the leader's MMAs) may still use them.
  __syncwarp();
  tc_fence_before();
  cluster_sync();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc2(tmem, 512);
  }
}

// ------------------------------------------------------- split-tail combine
// Combines the partial results of a split schedule, in a grid launched right
// after the attention kernel on the same stream (programmatic dependent
// launch: its set-up overlaps the attention kernel's end, griddep_wait holds
// it until every piece is written). Each (tail unit, query tile or CTA rank,
// 16-column group) is one CTA of 128 threads, one row per thread, the pieces'
// loads eight at a time in flight. (In the attention kernels, the last piece
// to finish combined a unit alone: one 8-GPU rank's shard of C5 at S=32768
// cuts every unit into ~10 pieces, and that combine -- ~640 KB of L2 reads by
// one CTA with two pieces in flight -- took ~10-20 us of a 66 us kernel.)
// Pieces are accumulated in CTA order, so the bits do not depend on which CTA
// finished first.
struct CombineParams {
  const float* ws_o;   // partial O slots, chunk-major [DPC/4][128 rows][4] fp32
  const float* ws_ml;  // partial (m, l) per slot row
  __half* o;
  int Sq, ld, D;       // output rows, row stride, valid columns per slot row
  int n_qb, unit_rows, tail_unit0, n_tiles, tail_ctas;
  long long total_steps;
  int pair;            // 1: D = 512 pair schedule (slot = (cluster, rank, piece))
};

template <int DPC>
__global__ void __launch_bounds__(128) attn_combine_kernel(const CombineParams c) {
  griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();
  const int rel = blockIdx.x;  // unit within the split tail
  const int t = blockIdx.y;    // query tile (D <= 128) or CTA rank (D = 512)
  const int cg = blockIdx.z;   // 16-column group
  const int row = threadIdx.x;
  if (16 * cg >= c.D) return;
  const int unit = c.tail_unit0 + rel;
  const int bh = unit / c.n_qb;
  const int rem = unit - bh * c.n_qb;
  int grow, col0 = 0;
  if (c.pair) {
    grow = ((rem >> 1) * 2 + t) * BM + row;
    col0 = 256 * (rem & 1);
  } else {
    if (t == 1 && c.unit_rows == BM) return;  // single-tile units
    grow = rem * c.unit_rows + t * BM + row;
  }
  if (grow >= c.Sq) return;
  const long long W = c.total_steps;
  const int GT = c.tail_ctas;
  const long long ubase = static_cast<long long>(rel) * c.n_tiles;
  const int c_lo = owner_cta(ubase, W, GT);
  const int np = owner_cta(ubase + c.n_tiles - 1, W, GT) - c_lo + 1;
  // slot row of piece k: range c_lo + k starts inside this unit (its first
  // tail segment, slot 0) iff floor(c * W / GT) >= ubase, i.e. c * W >= ubase * GT
  auto piece_row = [&](int k) -> long long {
    const long long c2 = c_lo + k;
    const long long which = (c2 * W >= ubase * GT) ? 0 : 1;
    const long long slot = c.pair ? (c2 * 2 + t) * 2 + which : (c2 * 2 + which) * 2 + t;
    return slot * BM + row;
  };
  auto piece_ml = [&](long long rb) -> float2 { return __ldcg(reinterpret_cast<const float2*>(c.ws_ml + rb * 2)); };
  float m_all = -INFINITY;
  for (int k = 0; k < np; ++k) m_all = fmaxf(m_all, piece_ml(piece_row(k)).x);
  float l_all = 0.f;
  for (int k = 0; k < np; ++k) {
    const float2 ml = piece_ml(piece_row(k));
    l_all = fmaf(ml.y, ex2_approx(ml.x - m_all), l_all);
  }
  const float inv = 1.f / l_all;
  float acc[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) acc[e] = 0.f;
  for (int k0 = 0; k0 < np; k0 += 8) {
    float4 v[8][4];
    float w[8];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int k = (k0 + kk < np) ? k0 + kk : k0;  // a duplicate load, never accumulated
      const long long rb = piece_row(k);
      w[kk] = ex2_approx(piece_ml(rb).x - m_all);
      const long long sl = rb / BM;
      const float* base = c.ws_o + sl * BM * DPC + (rb - sl * BM) * 4;
#pragma unroll
      for (int q = 0; q < 4; ++q) v[kk][q] = __ldcg(reinterpret_cast<const float4*>(base + (4 * cg + q) * BM * 4));
    }
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      if (k0 + kk < np) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[4 * q] = fmaf(v[kk][q].x, w[kk], acc[4 * q]);
          acc[4 * q + 1] = fmaf(v[kk][q].y, w[kk], acc[4 * q + 1]);
          acc[4 * q + 2] = fmaf(v[kk][q].z, w[kk], acc[4 * q + 2]);
          acc[4 * q + 3] = fmaf(v[kk][q].w, w[kk], acc[4 * q + 3]);
        }
      }
    }
  }
  __half* orow = c.o + (static_cast<long long>(bh) * c.Sq + grow) * c.ld + col0 + 16 * cg;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (16 * cg + 8 * h < c.D)
      *reinterpret_cast<uint4*>(orow + 8 * h) =
          make_uint4(pack_half2(acc[8 * h] * inv, acc[8 * h + 1] * inv), pack_half2(acc[8 * h + 2] * inv, acc[8 * h + 3] * inv),
                     pack_half2(acc[8 * h + 4] * inv, acc[8 * h + 5] * inv), pack_half2(acc[8 * h + 6] * inv, acc[8 * h + 7] * inv));
  }
}

// Self-test kernel: one thread waits on an mbarrier nothing arrives at.
__global__ void wait_timeout_selftest_kernel(unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    bwait(smem_u32(&bar), 0, 0, &abort_flag, timeout_ns, 0);
    // Complete the barrier's phase so nothing is left pending at exit.
    mbar_arrive(smem_u32(&bar));
  }
  __syncthreads();
}

}  // namespace fa

// ======================================================================= host

namespace {

thread_local int t_last_error = GFX906_B200_OK;

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// [B*H, S, D] fp16 tensor, boxes of 64 head-dim columns x `box_rows` rows, 128B swizzle.
bool make_map(CUtensorMap* m, const void* base, int D, int S, long long BH, int box_rows) {
  auto enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S),
                        static_cast<cuuint64_t>(BH)};
  cuuint64_t gstride[2] = {static_cast<cuuint64_t>(D) * 2,
                           static_cast<cuuint64_t>(S) * static_cast<cuuint64_t>(D) * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), gdim, gstride, box,
                   estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Transposed ("d-major") [B*H, D, S] fp16 tensor: the sequence is the
// innermost, contiguous dimension. Boxes of box_s positions x box_d head dims.
// 128B swizzle for MMA operand tiles (box_s = 64), none for the output store.
bool make_map_dmajor(CUtensorMap* m, const void* base, int D, int S, long long BH, int box_s, int box_d,
                     bool swizzle) {
  auto enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[3] = {static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(D),
                        static_cast<cuuint64_t>(BH)};
  cuuint64_t gstride[2] = {static_cast<cuuint64_t>(S) * 2,
                           static_cast<cuuint64_t>(S) * static_cast<cuuint64_t>(D) * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_s), static_cast<cuuint32_t>(box_d), 1};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), gdim, gstride, box,
                   estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct DeviceInfo {
  bool checked = false;
  bool sm100 = false;
  bool attrs_set = false;
  int num_sms = 0;
};
constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int check_device(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GFX906_B200_ECUDA;
  if (dev < 0 || dev >= kMaxDevices) return GFX906_B200_ENODEV;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& di = g_dev[dev];
  if (!di.checked) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return GFX906_B200_ECUDA;
    di.sm100 = (major == 10 && minor == 0);
    if (cudaDeviceGetAttribute(&di.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return GFX906_B200_ECUDA;
    di.checked = true;
  }
  if (!di.sm100) return GFX906_B200_ENODEV;
  if (!di.attrs_set) {
    if (cudaFuncSetAttribute(fa::attn_fwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             fa::Cfg<64>::SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(fa::attn_fwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             fa::Cfg<128>::SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(fa::attn_fwd_d512_pair_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             fa::Cfg512P::SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(fa::attn_fwd_d512_pair_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             fa::Cfg512P::SMEM_BYTES) != cudaSuccess)
      return GFX906_B200_ECUDA;
    di.attrs_set = true;
  }
  *dev_out = dev;
  return GFX906_B200_OK;
}

// Upper bound on the SMs a launch plans for (0: all of the device's), set by
// gfx906_b200_attn_set_sm_limit. A persistent grid of fewer CTAs than SMs
// leaves the rest to kernels on other streams, e.g. the NCCL collectives of
// the next or previous call of a sharded pipeline, which otherwise cannot
// start until the attention kernel ends.
std::atomic<int> g_sm_limit{0};

int device_sms(int dev) {
  const int n = g_dev[dev].num_sms > 0 ? g_dev[dev].num_sms : 1;
  const int lim = g_sm_limit.load(std::memory_order_relaxed);
  return (lim > 0 && lim < n) ? lim : n;
}

unsigned long long timeout_ns_from_env() {
  static unsigned long long v = [] {
    const char* e = getenv("GFX906_B200_WAIT_TIMEOUT_MS");
    unsigned long long ms = e ? strtoull(e, nullptr, 10) : 0ull;
    if (ms == 0ull) ms = 2000ull;
    return ms * 1000000ull;
  }();
  return v;
}


// Launch epochs tag the split counters (56 bits: never reused in practice).
// The sequence starts at a per-process, per-load pseudo-random point (clock,
// pid and this library's load address through the splitmix64 finaliser), so
// that two instances of the library -- two copies loaded in one process, or
// a workspace handed on from another user -- do not issue the same epochs
// and mistake each other's counters for their own.
unsigned long long seed_epoch() {
  uint64_t x = static_cast<uint64_t>(std::chrono::steady_clock::now().time_since_epoch().count());
  x ^= static_cast<uint64_t>(getpid()) << 40;
  x ^= static_cast<uint64_t>(reinterpret_cast<uintptr_t>(&seed_epoch));
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x & ((1ull << 56) - 1);
}
std::atomic<unsigned long long> g_epoch{seed_epoch()};
unsigned long long next_epoch() { return g_epoch.fetch_add(1) & ((1ull << 56) - 1); }

// Persistent schedule of attn_fwd_kernel (see SegIter in the kernel).
struct Plan {
  int G = 0;          // CTAs (at most one per SM)
  int split = 0;      // whole units, then a stream-K split of the tail units
  int tail_unit0 = 0;
  int tail_ctas = 0;
  int n_qb = 0, n_units = 0, n_tiles = 0;
  int unit_rows = 2 * fa::BM;
  long long total_steps = 0;  // steps of the tail
};
constexpr int kMinSplitSteps = 4;   // shortest key range a CTA gets in the tail
constexpr int kMinSplitTiles = 16;      // fewer units than SMs: split units of >= 16 key tiles
constexpr int kMinSplitTilesTail = 32;  // a partial last wave: split units of >= 32 key tiles

bool make_plan(long long BH, int Sq, int Skv, int num_sms, bool allow_split, Plan* pl) {
  pl->n_tiles = (Skv + fa::BN - 1) / fa::BN;
  const long long G = num_sms;
  const long long U256 = static_cast<long long>((Sq + 2 * fa::BM - 1) / (2 * fa::BM)) * BH;
  // Too few 256-row units for half the SMs, and units too short to split at
  // that size: one 128-row query tile per unit instead, twice the CTAs, and
  // each CTA's chain S -> softmax -> PV runs without the second tile's turns
  // in between (measured on B200: B1 H8 S1024 D64, 32 -> 64 units, 114 ->
  // 130 TFLOP/s, bit-identical). Such units are never split: cutting C1's
  // 8-key-tile units in two over 128 CTAs measured slower than 64 CTAs of
  // whole units (130 vs 138 TFLOP/s).
  const bool short_units = 2 * U256 <= G && (!allow_split || pl->n_tiles < kMinSplitTiles);
  pl->unit_rows = short_units ? fa::BM : 2 * fa::BM;
  pl->n_qb = (Sq + pl->unit_rows - 1) / pl->unit_rows;
  const long long U = static_cast<long long>(pl->n_qb) * BH;
  if (U > 0x7fffffffll) return false;
  pl->n_units = static_cast<int>(U);
  const long long waves = U / G;       // full waves of whole units
  const long long tail = U - waves * G;  // units left for a partial last wave
  // Split the tail's key range over the CTAs when whole units would leave SMs
  // idle in the last wave and units are long enough to amortise writing and
  // combining partial results: >= 16 key tiles when there are fewer units than
  // SMs, >= 32 otherwise. Measured on B200 (TFLOP/s,
  // whole -> split): 1x16384x131072 D64 (64 units) 292 -> 668; 1x131072^2 D64
  // (512 units, 1024 key tiles) 593 -> 688; 1x32768^2 D64 (128 units) 587 ->
  // 649; with the partial O stored chunk-major, B1 H8 S8192 D128 (64 key
  // tiles) 1072 -> 1150, B1 H24 S4096 D128 (32 key tiles) 1130 -> 1162, and
  // B2 H16 Sq4096 Skv1024 D128 (8 key tiles) 964 -> 935, which stays whole.
  const int min_tiles = waves == 0 ? kMinSplitTiles : kMinSplitTilesTail;
  pl->split = (allow_split && !short_units && tail > 0 && pl->n_tiles >= min_tiles) ? 1 : 0;
  if (pl->split) {
    pl->tail_unit0 = static_cast<int>(waves * G);
    pl->total_steps = tail * pl->n_tiles;
    long long gt = (pl->total_steps + kMinSplitSteps - 1) / kMinSplitSteps;
    if (gt > G) gt = G;
    // every CTA range is at least tail*T/gt >= T/(MAX_PIECES-1) steps long, so a
    // unit spans at most about MAX_PIECES ranges (a 16-unit shard of one long
    // head still gets all 148 SMs of a B200)
    if (gt > (fa::MAX_PIECES - 1) * tail) gt = (fa::MAX_PIECES - 1) * tail;
    pl->tail_ctas = static_cast<int>(gt);
    pl->G = static_cast<int>(waves > 0 ? G : gt);
  } else {
    pl->tail_unit0 = pl->n_units;
    pl->tail_ctas = 0;
    pl->total_steps = 0;
    pl->G = static_cast<int>(U < G ? U : G);
    if (pl->G < 1) pl->G = 1;
  }
  return true;
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Workspace of a split plan: [counters][partial (m, l)][partial O], slots of
// 128 rows per (CTA, piece, query tile), one counter per (tail unit, tile).
size_t workspace_bytes(const Plan& pl, int DP) {
  if (!pl.split) return 0;
  const size_t slots = static_cast<size_t>(pl.tail_ctas) * 2 * 2 * fa::BM;
  return align256(static_cast<size_t>(pl.n_units - pl.tail_unit0) * 2 * sizeof(unsigned long long)) +
         align256(slots * 2 * sizeof(float)) + slots * DP * sizeof(float);
}

// Who combines the pieces of a split D <= 128 plan: units cut into few pieces
// (fewer than 3 CTAs per tail unit on average) are combined in the attention
// kernel by the piece that finishes last, which overlaps the other CTAs' work
// (C2: 1145 vs 1075 TFLOP/s with the separate combine); units cut into many
// are combined by attn_combine_kernel, all of them in parallel (one 8-GPU
// rank's shard of C5 at S=32768, ~9 pieces per unit: 514 -> 601).
bool combine_in_kernel(const Plan& pl) {
  return static_cast<long long>(pl.tail_ctas) < 3ll * (pl.n_units - pl.tail_unit0);
}


// Launches a kernel with programmatic stream serialization: back-to-back
// calls on one stream then overlap the next call's launch and set-up with the
// end of this one (measured on B200: 5-6 us from the last CTA's exit to the
// next launch's first CTA without it). The kernels wait for the previous
// grid before their first global-memory access, so results and ordering are
// those of a plain launch. Falls back to a plain launch if the attribute is
// refused.
// cluster_x > 1 launches clusters of that many CTAs along x.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, int smem, cudaStream_t stream, int cluster_x,
               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster_x);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    cfg.numAttrs = 1;  // without programmatic serialization
    e = cudaLaunchKernelEx(&cfg, kernel, args...);
  }
  return (e == cudaSuccess && cudaGetLastError() == cudaSuccess) ? GFX906_B200_OK : GFX906_B200_ECUDA;
}

// Launches the combine of a split plan after the attention kernel.
int launch_combine(const Plan& pl, const fa::Params& prm, int dpc, int ld, int dvalid, int pair, cudaStream_t stream) {
  fa::CombineParams c{};
  c.ws_o = prm.ws_o;
  c.ws_ml = prm.ws_ml;
  c.o = prm.o;
  c.Sq = prm.Sq;
  c.ld = ld;
  c.D = dvalid;
  c.n_qb = pl.n_qb;
  c.unit_rows = pl.unit_rows;
  c.tail_unit0 = pl.tail_unit0;
  c.n_tiles = pl.n_tiles;
  c.tail_ctas = pl.tail_ctas;
  c.total_steps = pl.total_steps;
  c.pair = pair;
  const dim3 grid(static_cast<unsigned>(pl.n_units - pl.tail_unit0), 2, static_cast<unsigned>(dpc / 16));
  if (dpc == 64) return launch_pdl(fa::attn_combine_kernel<64>, grid, dim3(128), 0, stream, 1, c);
  if (dpc == 128) return launch_pdl(fa::attn_combine_kernel<128>, grid, dim3(128), 0, stream, 1, c);
  return launch_pdl(fa::attn_combine_kernel<256>, grid, dim3(128), 0, stream, 1, c);
}

template <int DP>
int launch_dp(const void* q, const void* k, const void* v, void* o, long long BH, int Sq, int Skv, int D,
              float scale, void* ws, size_t ws_size, int dev, cudaStream_t stream) {
  Plan pl;
  if (!make_plan(BH, Sq, Skv, device_sms(dev), ws != nullptr, &pl)) return GFX906_B200_EINVAL;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, q, D, Sq, BH, fa::BM) || !make_map(&mk, k, D, Skv, BH, fa::BN) ||
      !make_map(&mv, v, D, Skv, BH, fa::BN))
    return GFX906_B200_ECUDA;
  fa::Params prm{};
  prm.Sq = Sq;
  prm.Skv = Skv;
  prm.D = D;
  prm.bh_offset = 0;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.timeout_ns = timeout_ns_from_env();
  prm.n_qb = pl.n_qb;
  prm.unit_rows = pl.unit_rows;
  prm.n_units = pl.n_units;
  prm.n_tiles = pl.n_tiles;
  prm.split = pl.split;
  prm.tail_unit0 = pl.tail_unit0;
  prm.tail_ctas = pl.tail_ctas;
  prm.total_steps = pl.total_steps;
  prm.o = static_cast<__half*>(o);
  if (pl.split) {
    const size_t need = workspace_bytes(pl, DP);
    if (ws_size < need || (reinterpret_cast<uintptr_t>(ws) & 255u)) return GFX906_B200_EINVAL;
    uint8_t* base = static_cast<uint8_t*>(ws);
    const size_t slots = static_cast<size_t>(pl.tail_ctas) * 2 * 2 * fa::BM;
    prm.ws_cnt = reinterpret_cast<unsigned long long*>(base);
    base += align256(static_cast<size_t>(pl.n_units - pl.tail_unit0) * 2 * sizeof(unsigned long long));
    prm.epoch = next_epoch();
    prm.ws_ml = reinterpret_cast<float*>(base);
    base += align256(slots * 2 * sizeof(float));
    prm.ws_o = reinterpret_cast<float*>(base);
    prm.combine = combine_in_kernel(pl) ? 1 : 0;
  }
  const int rc = launch_pdl(fa::attn_fwd_kernel<DP>, dim3(pl.G), dim3(fa::NUM_THREADS), fa::Cfg<DP>::SMEM_BYTES,
                            stream, 1, mq, mk, mv, prm);
  if (rc != GFX906_B200_OK || !pl.split || prm.combine) return rc;
  return launch_combine(pl, prm, DP, D, D, 0, stream);
}

// Persistent schedule of attn_fwd_d512_pair_kernel: units are (batch x head,
// query-tile pair, head-dim half), one cluster of two CTAs per SM pair.
// Whole units first; with a workspace, the last partial wave's key range is
// split over the clusters (units of >= kMinSplitTiles512 key tiles) when
// there are fewer units than clusters or the partial wave is at most half
// full. Measured on B200 (TFLOP/s, whole -> split): one 8-GPU rank's row shard
// of C4 (1x4x512x4096, 16 units) 217 -> 307, a 4-GPU shard 442 -> 551; C4
// itself (128 units, a partial wave of 54 on 74 clusters) 877 -> 849, so it
// runs whole units.
constexpr int kMinSplitTiles512 = 8;

bool make_plan512(long long BH, int Sq, int Skv, int num_sms, bool allow_split, Plan* pl) {
  const long long npairs = ((Sq + fa::BM - 1) / fa::BM + 1) / 2;
  pl->n_qb = static_cast<int>(2 * npairs);  // units per (batch, head)
  pl->unit_rows = 2 * fa::BM;
  pl->n_tiles = (Skv + fa::BN - 1) / fa::BN;
  const long long U = 2 * npairs * BH;
  if (U > 0x7fffffffll) return false;
  pl->n_units = static_cast<int>(U);
  const long long G = num_sms / 2 > 0 ? num_sms / 2 : 1;  // clusters
  const long long waves = U / G;
  const long long tail = U - waves * G;
  pl->split = (allow_split && tail > 0 && pl->n_tiles >= kMinSplitTiles512 && (waves == 0 || 2 * tail <= G)) ? 1 : 0;
  if (pl->split) {
    pl->tail_unit0 = static_cast<int>(waves * G);
    pl->total_steps = tail * pl->n_tiles;
    long long gt = (pl->total_steps + kMinSplitSteps - 1) / kMinSplitSteps;
    if (gt > G) gt = G;
    if (gt > (fa::MAX_PIECES - 1) * tail) gt = (fa::MAX_PIECES - 1) * tail;
    pl->tail_ctas = static_cast<int>(gt);
    pl->G = static_cast<int>(waves > 0 ? G : gt);
  } else {
    pl->tail_unit0 = pl->n_units;
    pl->tail_ctas = 0;
    pl->total_steps = 0;
    pl->G = static_cast<int>(U < G ? U : G);
  }
  return true;
}

// Workspace of a split D = 512 plan: [partial (m, l)][partial O], slots of
// 128 rows x 256 fp32 per (cluster, rank, piece).
size_t workspace_bytes512(const Plan& pl) {
  if (!pl.split) return 0;
  const size_t slots = static_cast<size_t>(pl.tail_ctas) * 2 * 2 * fa::BM;
  return align256(slots * 2 * sizeof(float)) + slots * fa::Cfg512P::DH * sizeof(float);
}

// D = 512 on CTA pairs: grid x = 2 x clusters, clusters of 2. DMAJOR: the
// transposed layout, whole units only (the workspace is ignored).
template <bool DMAJOR>
int launch_d512_pair(const void* q, const void* k, const void* v, void* o, long long BH, int Sq, int Skv,
                     float scale, void* ws, size_t ws_size, int dev, cudaStream_t stream) {
  if (DMAJOR) ws = nullptr;
  Plan pl;
  if (!make_plan512(BH, Sq, Skv, device_sms(dev), ws != nullptr, &pl)) return GFX906_B200_EINVAL;
  if (BH > 0x7fffffffll) return GFX906_B200_EINVAL;
  CUtensorMap mq, mk, mv, mo;
  if (DMAJOR) {
    if (!make_map_dmajor(&mq, q, 512, Sq, BH, 64, 256, true) || !make_map_dmajor(&mk, k, 512, Skv, BH, 64, 256, true) ||
        !make_map_dmajor(&mv, v, 512, Skv, BH, 64, 128, true) ||
        !make_map_dmajor(&mo, o, 512, Sq, BH, fa::BM, fa::Cfg512P::DH, false))
      return GFX906_B200_ECUDA;
  } else if (!make_map(&mq, q, 512, Sq, BH, fa::BM) || !make_map(&mk, k, 512, Skv, BH, fa::BN / 2) ||
             !make_map(&mv, v, 512, Skv, BH, fa::BN) || !make_map(&mo, o, 512, Sq, BH, fa::BM)) {
    return GFX906_B200_ECUDA;
  }
  fa::Params prm{};
  prm.Sq = Sq;
  prm.Skv = Skv;
  prm.D = 512;
  prm.bh_offset = 0;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.timeout_ns = timeout_ns_from_env();
  prm.n_qb = pl.n_qb;
  prm.unit_rows = pl.unit_rows;
  prm.n_units = pl.n_units;
  prm.n_tiles = pl.n_tiles;
  prm.split = pl.split;
  prm.tail_unit0 = pl.tail_unit0;
  prm.tail_ctas = pl.tail_ctas;
  prm.total_steps = pl.total_steps;
  prm.o = static_cast<__half*>(o);
  if (pl.split) {
    const size_t need = workspace_bytes512(pl);
    if (ws_size < need || (reinterpret_cast<uintptr_t>(ws) & 255u)) return GFX906_B200_EINVAL;
    uint8_t* base = static_cast<uint8_t*>(ws);
    const size_t slots = static_cast<size_t>(pl.tail_ctas) * 2 * 2 * fa::BM;
    prm.ws_ml = reinterpret_cast<float*>(base);
    base += align256(slots * 2 * sizeof(float));
    prm.ws_o = reinterpret_cast<float*>(base);
  }
  const int rc = launch_pdl(fa::attn_fwd_d512_pair_kernel<DMAJOR>, dim3(2 * static_cast<unsigned>(pl.G)),
                            dim3(fa::Cfg512P::THREADS), fa::Cfg512P::SMEM_BYTES, stream, 2, mq, mk, mv, mo, prm);
  if (rc != GFX906_B200_OK || !pl.split) return rc;
  return launch_combine(pl, prm, fa::Cfg512P::DH, 512, fa::Cfg512P::DH, 1, stream);
}

// Argument checks shared by every entry point. Returns OK and sets *skip when
// there is nothing to compute.
int check_args(const void* q, const void* k, const void* v, const void* o, int B, int H, int Sq, int Skv,
               int D, bool* skip) {
  *skip = false;
  if (B < 0 || H < 0 || Sq < 0 || Skv < 0) return GFX906_B200_EINVAL;
  if (!((D >= 8 && D <= 64 && D % 8 == 0) || D == 128 || D == 512)) return GFX906_B200_EHEADDIM;
  const long long BH = static_cast<long long>(B) * H;
  if (BH == 0 || Sq == 0) {
    *skip = true;
    return GFX906_B200_OK;
  }
  if (BH > (1ll << 31) || static_cast<long long>(Sq) * D * 2 * BH >= (1ll << 40) ||
      static_cast<long long>(Skv) * D * 2 * BH >= (1ll << 40))
    return GFX906_B200_EINVAL;
  // k and v may be empty (and then null) when Skv == 0; q and o hold data here.
  if (!q || !o || (Skv > 0 && (!k || !v))) return GFX906_B200_EINVAL;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(o)) & 15u)
    return GFX906_B200_EALIGN;
  return GFX906_B200_OK;
}

int attn_launch_impl(const void* q, const void* k, const void* v, void* o, int B, int H, int Sq, int Skv,
                     int D, float scale, void* ws, size_t ws_size, cudaStream_t stream) {
  bool skip = false;
  int rc = check_args(q, k, v, o, B, H, Sq, Skv, D, &skip);
  if (rc != GFX906_B200_OK || skip) return rc;
  const long long BH = static_cast<long long>(B) * H;
  int dev = 0;
  rc = check_device(&dev);
  if (rc != GFX906_B200_OK) return rc;
  if (Skv == 0) {
    // softmax over an empty key set: defined here as a zero output.
    if (cudaMemsetAsync(o, 0, static_cast<size_t>(BH) * Sq * D * 2, stream) != cudaSuccess)
      return GFX906_B200_ECUDA;
    return GFX906_B200_OK;
  }
  if (D == 128) return launch_dp<128>(q, k, v, o, BH, Sq, Skv, D, scale, ws, ws_size, dev, stream);
  if (D <= 64) return launch_dp<64>(q, k, v, o, BH, Sq, Skv, D, scale, ws, ws_size, dev, stream);
  return launch_d512_pair<false>(q, k, v, o, BH, Sq, Skv, scale, ws, ws_size, dev, stream);
}

}  // namespace

extern "C" {

int gfx906_b200_attn_launch(const void* q, const void* k, const void* v, void* o, int B, int H, int Sq,
                            int Skv, int D, float scale, cudaStream_t stream) {
  const int rc = attn_launch_impl(q, k, v, o, B, H, Sq, Skv, D, scale, nullptr, 0, stream);
  t_last_error = rc;
  return rc;
}

int gfx906_b200_attn_launch_dmajor(const void* q, const void* k, const void* v, void* o, int B, int H, int Sq,
                                   int Skv, int D, float scale, cudaStream_t stream) {
  bool skip = false;
  int rc = check_args(q, k, v, o, B, H, Sq, Skv, D, &skip);
  if (rc == GFX906_B200_OK && !skip) {
    if (D != 512) {
      rc = GFX906_B200_EHEADDIM;
    } else if (Sq % 8 != 0 || Skv % 8 != 0) {
      rc = GFX906_B200_EALIGN;  // every [D][S] row must start on 16 bytes for TMA
    } else {
      int dev = 0;
      rc = check_device(&dev);
      if (rc == GFX906_B200_OK) {
        const long long BH = static_cast<long long>(B) * H;
        if (Skv == 0) {
          rc = cudaMemsetAsync(o, 0, static_cast<size_t>(BH) * Sq * D * 2, stream) == cudaSuccess
                   ? GFX906_B200_OK
                   : GFX906_B200_ECUDA;
        } else {
          rc = launch_d512_pair<true>(q, k, v, o, BH, Sq, Skv, scale, nullptr, 0, dev, stream);
        }
      }
    }
  }
  t_last_error = rc;
  return rc;
}

size_t gfx906_b200_attn_workspace_size(int B, int H, int Sq, int Skv, int D) {
  bool skip = false;
  const int probe = 16;  // any aligned non-null value: only sizes are checked here
  const void* fake = reinterpret_cast<const void*>(static_cast<uintptr_t>(probe));
  if (check_args(fake, fake, fake, fake, B, H, Sq, Skv, D, &skip) != GFX906_B200_OK || skip) return 0;
  if (Skv == 0) return 0;
  int dev = 0;
  if (check_device(&dev) != GFX906_B200_OK) return 0;
  Plan pl;
  if (D == 512) {
    if (!make_plan512(static_cast<long long>(B) * H, Sq, Skv, device_sms(dev), true, &pl)) return 0;
    return workspace_bytes512(pl);
  }
  if (!make_plan(static_cast<long long>(B) * H, Sq, Skv, device_sms(dev), true, &pl)) return 0;
  return workspace_bytes(pl, D == 128 ? 128 : 64);
}

int gfx906_b200_attn_plan(int B, int H, int Sq, int Skv, int D, int with_workspace, int num_sms, int* out4) {
  if (!out4) return GFX906_B200_EINVAL;
  bool skip = false;
  const void* fake = reinterpret_cast<const void*>(static_cast<uintptr_t>(16));
  int rc = check_args(fake, fake, fake, fake, B, H, Sq, Skv, D, &skip);
  if (rc != GFX906_B200_OK) return rc;
  out4[0] = out4[1] = out4[2] = out4[3] = 0;
  if (skip || Skv == 0) return GFX906_B200_OK;  // nothing is launched
  if (num_sms <= 0) {
    int dev = 0;
    rc = check_device(&dev);
    if (rc != GFX906_B200_OK) return rc;
    num_sms = device_sms(dev);
  }
  const long long BH = static_cast<long long>(B) * H;
  Plan pl;
  if (D == 512) {
    // CTAs (2 per cluster); unit_rows = query rows of a unit (a pair of tiles)
    if (!make_plan512(BH, Sq, Skv, num_sms, with_workspace != 0, &pl)) return GFX906_B200_EINVAL;
    out4[0] = 2 * pl.G;
    out4[1] = pl.split ? 2 : 0;  // D = 512 pieces are always combined by attn_combine_kernel
    out4[2] = 2 * pl.tail_ctas;
    out4[3] = pl.unit_rows;
    return GFX906_B200_OK;
  }
  if (!make_plan(BH, Sq, Skv, num_sms, with_workspace != 0, &pl)) return GFX906_B200_EINVAL;
  out4[0] = pl.G;
  out4[1] = pl.split ? (combine_in_kernel(pl) ? 1 : 2) : 0;
  out4[2] = pl.tail_ctas;
  out4[3] = pl.unit_rows;
  return GFX906_B200_OK;
}

int gfx906_b200_internal_set_last_error(int status) {
  t_last_error = status;
  return status;
}

int gfx906_b200_attn_launch_ws(const void* q, const void* k, const void* v, void* o, int B, int H, int Sq,
                               int Skv, int D, float scale, void* workspace, size_t workspace_bytes,
                               cudaStream_t stream) {
  const int rc = attn_launch_impl(q, k, v, o, B, H, Sq, Skv, D, scale, workspace, workspace_bytes, stream);
  t_last_error = rc;
  return rc;
}

void launch(const void* q, const void* k, const void* v, void* o, int B, int H, int Sq, int Skv, int D,
            float scale, cudaStream_t stream) {
  (void)gfx906_b200_attn_launch(q, k, v, o, B, H, Sq, Skv, D, scale, stream);
}

int gfx906_b200_attn_last_error(void) { return t_last_error; }

int gfx906_b200_attn_set_sm_limit(int sms) { return g_sm_limit.exchange(sms > 0 ? sms : 0); }

const char* gfx906_b200_attn_error_string(int status) {
  switch (status) {
    case GFX906_B200_OK: return "ok";
    case GFX906_B200_EINVAL: return "invalid argument (negative size, null pointer or size overflow)";
    case GFX906_B200_EHEADDIM: return "unsupported head_dim (need <=64 and a multiple of 8, 128, or 512)";
    case GFX906_B200_EALIGN: return "q, k, v and o must be 16-byte aligned";
    case GFX906_B200_ENODEV: return "current CUDA device is not an sm_100 (B200) GPU";
    case GFX906_B200_ECUDA: return "a CUDA runtime or driver call failed";
    case GFX906_B200_ETIMEOUT: return "a kernel wait timed out (device status word set)";
    case GFX906_B200_ENOSPACE: return "the call needs more scratch than the allocation-free entry point's array holds";
    default: return "unknown status";
  }
}

int gfx906_b200_attn_device_status(int reset) {
  if (cudaDeviceSynchronize() != cudaSuccess) return GFX906_B200_ECUDA;
  unsigned int st = 0;
  if (cudaMemcpyFromSymbol(&st, fa::g_status, sizeof(st)) != cudaSuccess) return GFX906_B200_ECUDA;
  if (reset) {
    const unsigned int zero = 0;
    int zeros[6] = {0, 0, 0, 0, 0, 0};
    if (cudaMemcpyToSymbol(fa::g_status, &zero, sizeof(zero)) != cudaSuccess ||
        cudaMemcpyToSymbol(fa::g_timeout_info, zeros, sizeof(zeros)) != cudaSuccess)
      return GFX906_B200_ECUDA;
  }
  return st ? GFX906_B200_ETIMEOUT : GFX906_B200_OK;
}

int gfx906_b200_attn_timeout_info(int* out6) {
  if (!out6) return GFX906_B200_EINVAL;
  if (cudaDeviceSynchronize() != cudaSuccess) return GFX906_B200_ECUDA;
  if (cudaMemcpyFromSymbol(out6, fa::g_timeout_info, 6 * sizeof(int)) != cudaSuccess) return GFX906_B200_ECUDA;
  return GFX906_B200_OK;
}

int gfx906_b200_attn_selftest_wait_timeout(unsigned long long timeout_ns, cudaStream_t stream) {
  int dev = 0;
  int rc = check_device(&dev);
  if (rc != GFX906_B200_OK) return rc;
  fa::wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(timeout_ns);
  return cudaGetLastError() == cudaSuccess ? GFX906_B200_OK : GFX906_B200_ECUDA;
}

double gfx906_b200_attn_flops(int B, int H, int Sq, int Skv, int D) {
  return 4.0 * B * H * static_cast<double>(Sq) * Skv * D;
}

}  // extern "C"
