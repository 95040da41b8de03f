// fo_kernel.cuh -- the persistent, warp-specialised tcgen05 kernel behind every operator
// of the library: gemm, gemm+bias(+act), gemm+bias+LayerNorm and conv2d (implicit GEMM).
//
// One CTA per SM loops over 128 x BN output tiles.  Warp roles:
//   producer  : GEMM -- one thread issues TMA loads of A (128 x 64) and B (BN x 64) per
//               k-block into a `stages`-deep shared-memory ring;
//               conv -- a 128-thread warpgroup gathers the im2col rows of A with 16-byte
//               cp.async (zero-fill gives the padding) while one thread TMA-loads the
//               weight tile.
//   mma       : one thread issues tcgen05.mma (M=128, N=BN, K=16) into one of two TMEM
//               accumulators (2 x BN fp32 columns), so the epilogue of tile i overlaps
//               the mainloop of tile i+1.
//   epilogue  : eight warps (two per TMEM lane quarter, one per column half) read the
//               accumulator with tcgen05.ld, apply bias / activation in fp32, convert,
//               stage 32 x 128 B blocks in 128B-swizzled shared memory and write them
//               with TMA stores (16-bit 64-column tiles store from registers).
//               For LayerNorm each thread owns one output row, so exact per-row
//               (mean, M2) of the fp32 tile slice is a register reduction; the slice
//               is stored centred on a shift and a row pass (next on the stream:
//               fo_ln_rows_kernel or fo_ln_normalize_kernel) merges the slices'
//               statistics (Chan et al.) and normalises.
// Every wait is bounded (mbar_wait); a wait that runs out records FO_ETIMEOUT in the
// device status word, raises a CTA-local abort flag, drains its in-flight copies and
// returns.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fo_ptx.cuh"

namespace fo {

enum : int { DT_F16 = 0, DT_BF16 = 1, DT_F32 = 2 };
enum : int { ACT_NONE = 0, ACT_RELU = 1, ACT_GELU_TANH = 2, ACT_GELU_ERF = 3 };

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 16-bit elements = one 128-byte swizzle row
constexpr int kAStageBytes = kBM * kBK * 2;
// Eight epilogue warps: two per TMEM lane quarter (a warp may read only lanes
// 32 * (warp % 4) ..), each taking half of the tile's columns, so the per-element work of
// the epilogue (activation, statistics, conversion) is spread over two warps per SM
// sub-partition.  Each warp stages its stores in one 4 KB block (32 rows x 128 B).
constexpr int kEpiWarps = 8;
constexpr int kEpiBufBytes = 32 * 128;
constexpr int kEpiBytes = kEpiWarps * kEpiBufBytes;
constexpr int kMiscBytes = 1536;
constexpr int kMaxStages = 8;
// One-kernel LayerNorm: most units a slice may wait, after its own, for its rows'
// statistics (the host takes the two-kernel path when the tile raster needs more).
constexpr int kLnMaxDefer = 3;
__host__ __device__ constexpr int ln_defer_for(int span, int ncl) {
  return ncl <= 0 ? 1 << 20 : (span + ncl - 1) / ncl < 1 ? 1 : (span + ncl - 1) / ncl;
}

// Status codes written into the device status word (first writer wins).
constexpr int kStatusTimeout = 5;

struct KParams {
  int M, N, K;
  int tiles_m, tiles_n, num_tiles, k_blocks;
  int group_m;
  int stages;
  int ab_bf16;
  int b_mn;
  int has_bias;
  const void* bias;
  const void* gamma;
  const void* beta;
  int vec_dtype;
  float eps;
  float4* ln_stats;  // [tiles_n][M] (mean, M2, shift, 0) of each row over one N tile
  const void* residual;  // residual LayerNorm: [M, N] rows added before normalising
  long long ldr;
  void* out;
  long long ldo;
  int* status;  // [0] = code, [1] = where, [2] = block
  unsigned long long timeout_ns;
  // implicit-GEMM conv geometry (NHWC)
  const void* x;
  int H, W, C, OH, OW, KH, KW, stride, pad, dil, c_blocks;
  int conv_tma;  // 1: A tiles by TMA im2col loads (tmA); 0: cp.async gather
  // direct conv (fo_direct_conv_kernel): input rows padded to pitch P positions, Hp padded
  // rows per image, nR rows per pixel slot, pslots slots, nimg images; a tile is rpt
  // output rows (rpt * P positions) of one image, tpi tiles per image
  int P, Hp, nR, pslots, nimg, rpt, tpi;
  // k-blocks (64-wide K slices) per pipeline stage: 1 or 2 (block_k 128).  Two per stage
  // halve the barrier waits, fences and commits the single MMA-issuing thread spends per
  // MMA (8 MMAs per wait / commit instead of 4).
  int kps;
  // work units: units [0, dp_units) are whole tiles; the remaining tiles are split along K
  // into `split` parts of kb_per_part k-blocks, reduced through split_ws / split_cnt.
  int num_units, dp_units, split, kb_per_part;
  // 1: the split tiles are the raster's first tiles and their parts run first (unit
  // u < num_units - dp_units is split part u, whole tile w the unit after them), so their
  // partial-sum exchange overlaps the whole tiles' mainloops instead of ending the grid.
  int tail_first;
  // conv BatchNorm epilogues (inference form): per output channel f, with acc rounded to
  // the input dtype first, y = (acc - mean[f]) * rsqrt(var[f] + bn_eps) * gamma[f] + beta[f], var clamped at 0
  // when bn_mode == 2; then + add_src[pixel][f] when add_src is set; then ACT.
  int bn_mode;  // 0 none, 1 BN, 2 BN with var clamped at 0
  float bn_eps;
  const void *bn_gamma, *bn_beta, *bn_mean, *bn_var;  // vec_dtype
  const void* add_src;  // [M pixels, N] of the output dtype, row stride ld_add (or null)
  long long ld_add;
  // cluster split (csplit = s >= 2): the s parts of a tile are the CTAs of one cluster
  // (unit = tile * s + cluster rank, one unit per CTA); each CTA owns the 32 x 32 chunks
  // g (= quarter * BN/32 + column chunk) with g % s == rank, receives the other parts'
  // fp32 partials of them into shared memory (st.async) and runs their epilogue.
  int csplit;
  // [split slot][part][row quarter][column half][BN/2 columns][32 rows] fp32 partials:
  // one contiguous block per (part, epilogue warp)
  float* split_ws;
  int* split_cnt;   // [split slot][4 row quarters] arrival counters, self-resetting
                    // (a slot is a split tile's 128 rows: two per tile for CTA pairs)
  // One-kernel LayerNorm (ln_fused = 1; launched cooperatively, every CTA resident): each
  // epilogue warp publishes the (mean, M2) of its row slice to ln_st2[slice][row] and
  // counts itself into ln_cnt[row / 32]; the arrival that completes the 32 rows merges
  // their statistics into ln_fin; some units later the same warp reads its stored slice
  // back and normalises it in place.  ln_fused = 2: the warp keeps its slice in the TMEM
  // accumulator instead (nothing stored early), waits at the same unit for the merged
  // statistics and normalises straight from TMEM before releasing the accumulator; this
  // needs every row block's tiles within ln_span < (units per wave) of each other.
  // ln_cnt holds 2 x ln_groups int32 (arrivals, then finished normalisers),
  // zero at launch and reset to zero by the last normaliser of each group.
  int ln_fused;
  int ln_span;    // largest unit distance between two tiles of one row block
  int ln_groups;  // ceil(M / 32)
  int* ln_cnt;
  float2* ln_st2;  // [2 x tiles_n slices][M] (mean, M2) of each row slice
  float2* ln_fin;  // [M] (mean, rstd) of each row, written by its group's last arrival
};

__host__ __device__ constexpr int b_stage_bytes(int bn) { return bn * kBK * 2; }
// Cluster split: a received 32 x 32 fp32 chunk is stored as 32 rows of 144 bytes (128 of
// data, padded so that 16-byte accesses by consecutive rows hit distinct banks).
constexpr int kRedRowBytes = 144;
constexpr int kRedChunkBytes = 32 * kRedRowBytes;
__host__ __device__ constexpr int csplit_owned_max(int bn, int s) { return (4 * (bn / 32) + s - 1) / s; }
// Receive area of a cluster-split CTA: (s - 1) senders x its owned chunks.
__host__ __device__ constexpr int csplit_recv_bytes(int bn, int s) {
  return s > 1 ? (s - 1) * csplit_owned_max(bn, s) * kRedChunkBytes : 0;
}
// The epilogue region holds the store staging or, in a cluster split (whose epilogue
// stores from registers), the receive area.
__host__ __device__ constexpr int epi_region_bytes(int bn, int csplit) {
  return csplit_recv_bytes(bn, csplit) > kEpiBytes ? csplit_recv_bytes(bn, csplit) : kEpiBytes;
}
// pair: CTA-pair kernel (block_m 256), where each CTA holds half of the B tile.
// kps: k-blocks per stage (block_k / 64).  csplit: parts of a cluster split (0 or 1: none).
__host__ __device__ constexpr int smem_bytes_for(int bn, int stages, bool pair = false, int kps = 1, int csplit = 0) {
  return 1024 + stages * kps * (kAStageBytes + b_stage_bytes(pair ? bn / 2 : bn)) + epi_region_bytes(bn, csplit) +
         kMiscBytes;
}

__device__ __forceinline__ void record_error(const KParams& p, int code, int where) {
  if (atomicCAS(p.status, 0, code) == 0) {
    p.status[1] = where;
    p.status[2] = static_cast<int>(blockIdx.x);
  }
}

__device__ __forceinline__ float load_vec(const void* ptr, int dt, int i);

// Per-channel affine of the epilogue: y = acc * scale + shift.  Bias: (1, bias[f]);
// BatchNorm: scale = gamma * rsqrt(var + eps), shift = beta - mean * scale (var clamped
// at 0 for bn_mode 2, as the reference's conv_bn_add_relu does).
__device__ __forceinline__ float2 channel_affine(const KParams& p, int f) {
  if (f >= p.N) return make_float2(1.f, 0.f);
  if (p.bn_mode) {
    float var = load_vec(p.bn_var, p.vec_dtype, f);
    if (p.bn_mode == 2) var = fmaxf(var, 0.f);
    const float sc = load_vec(p.bn_gamma, p.vec_dtype, f) * rsqrtf(var + p.bn_eps);
    return make_float2(sc, fmaf(-load_vec(p.bn_mean, p.vec_dtype, f), sc, load_vec(p.bn_beta, p.vec_dtype, f)));
  }
  return make_float2(1.f, p.has_bias ? load_vec(p.bias, p.vec_dtype, f) : 0.f);
}

// The conv result rounded to the input dtype, as the reference's BatchNorm operators see
// it (their fp16 F.conv2d / fp16 out_shared tile) before applying the BatchNorm.
__device__ __forceinline__ float round_in(float v, int ab_bf16) {
  return ab_bf16 ? __bfloat162float(__float2bfloat16_rn(v)) : __half2float(__float2half_rn(v));
}

__device__ __forceinline__ float load_vec(const void* ptr, int dt, int i) {
  if (dt == DT_F32) return __ldg(reinterpret_cast<const float*>(ptr) + i);
  const unsigned short raw = __ldg(reinterpret_cast<const unsigned short*>(ptr) + i);
  if (dt == DT_BF16) return __bfloat162float(__ushort_as_bfloat16(raw));
  return __half2float(__ushort_as_half(raw));
}

// erf(z) by Abramowitz & Stegun, Handbook of Mathematical Functions, 7.1.28:
// erf(z) = 1 - (1 + a1 z + a2 z^2 + a3 z^3 + a4 z^4 + a5 z^5 + a6 z^6)^-16 for z >= 0,
// |error| <= 3e-7 (2.7e-6 evaluated in fp32 with the approximate reciprocal below; the
// GELU built on it stays within 9e-7 of the exact one), odd in z.  One reciprocal, six
// FMAs and four squarings, branch-free: the special-function unit runs one op per
// element instead of the two of 7.1.26 (reciprocal and exponential), which made GELU-erf
// the slowest epilogue (a 128 x 256 tile: 8.2 us against 4.1 for the tanh form).  For
// large z the polynomial overflows to inf, its reciprocal is 0 and erf is 1.
__device__ __forceinline__ float erf_as7128(float z) {
  const float az = fabsf(z);
  float p = fmaf(fmaf(fmaf(fmaf(fmaf(4.30638e-5f, az, 2.765672e-4f), az, 1.520143e-4f), az, 9.2705272e-3f), az,
                      4.22820123e-2f),
                 az, 7.05230784e-2f);
  p = fmaf(p, az, 1.0f);
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(p));
  r *= r;  // r^2
  r *= r;  // r^4
  r *= r;  // r^8
  r *= r;  // r^16
  return copysignf(1.0f - r, z);
}

template <int ACT>
__device__ __forceinline__ float apply_act(float x) {
  if constexpr (ACT == ACT_RELU) {
    return fmaxf(x, 0.0f);
  } else if constexpr (ACT == ACT_GELU_TANH) {
    // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))  -- end2end.py:37-38 new_gelu
    const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
    return 0.5f * x * (1.0f + t);
  } else if constexpr (ACT == ACT_GELU_ERF) {
    return 0.5f * x * (1.0f + erf_as7128(x * 0.7071067811865476f));
  } else {
    return x;
  }
}

template <int DT>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (DT == DT_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}
template <int DT>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
  if constexpr (DT == DT_BF16) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
    return __bfloat1622float2(h);
  } else {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
  }
}

// Eight consecutive vector elements i..i+7 (16-byte aligned) as fp32.
__device__ __forceinline__ void load_vec8(const void* ptr, int dt, int i, float (&f)[8]) {
  if (dt == DT_F32) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(ptr) + i / 4);
    const float4 b = __ldg(reinterpret_cast<const float4*>(ptr) + i / 4 + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    return;
  }
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(ptr) + i / 8);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 v = dt == DT_BF16 ? unpack2<DT_BF16>(w[e]) : unpack2<DT_F16>(w[e]);
    f[2 * e] = v.x;
    f[2 * e + 1] = v.y;
  }
}

// Forces every later use of r[] to follow tcgen05.wait::ld.
__device__ __forceinline__ void tc_wait_ld_regs(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// Orders uses of registers filled by an earlier tcgen05.ld after a tcgen05.wait::ld
// issued for another load (volatile asm statements keep their relative order).
__device__ __forceinline__ void tc_pin_regs(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31]));
}

__device__ __forceinline__ void tile_coords(const KParams& p, int t, int& tm, int& tn) {
  if (p.group_m <= 0) {
    tm = t / p.tiles_n;
    tn = t - tm * p.tiles_n;
    return;
  }
  const int per_group = p.group_m * p.tiles_n;
  const int g = t / per_group;
  const int r = t - g * per_group;
  const int first_m = g * p.group_m;
  const int gm = min(p.group_m, p.tiles_m - first_m);
  tm = first_m + r % gm;
  tn = r / gm;
}

struct Unit {
  int tm, tn, kb0, kb1;
  int st;    // index of the split tile, or -1 for a whole tile
  int part;  // K part of a split tile
};

__device__ __forceinline__ Unit unit_of(const KParams& p, int u) {
  Unit r;
  int tile;
  int whole0 = 0, split0 = p.dp_units;  // first tile of the whole / split tiles
  if (p.tail_first) {
    // split tiles are the raster's first tiles and their parts the first units, so the
    // schedule walks the raster from its start (L2 reuse as without a split)
    const int parts = p.num_units - p.dp_units;
    if (u < parts) {
      u += p.dp_units;
      split0 = 0;
    } else {
      u -= parts;
      whole0 = parts / p.split;
    }
  }
  if (u < p.dp_units) {
    tile = whole0 + u;
    r.kb0 = 0;
    r.kb1 = p.k_blocks;
    r.st = -1;
    r.part = 0;
  } else {
    const int v = u - p.dp_units;
    r.st = v / p.split;
    r.part = v - r.st * p.split;
    tile = split0 + r.st;
    if (p.csplit > 1) {
      // cluster split: the tile's stages (kps k-blocks each) spread evenly over the
      // parts, so no part is empty while parts <= stages
      const int nst = (p.k_blocks + p.kps - 1) / p.kps;
      r.kb0 = min(p.k_blocks, (r.part * nst / p.split) * p.kps);
      r.kb1 = min(p.k_blocks, ((r.part + 1) * nst / p.split) * p.kps);
    } else {
      r.kb0 = r.part * p.kb_per_part;
      r.kb1 = min(p.k_blocks, r.kb0 + p.kb_per_part);
    }
  }
  tile_coords(p, tile, r.tm, r.tn);
  return r;
}

// Chan et al. parallel merge of (count, mean, M2).
__device__ __forceinline__ void chan_merge(float& cnt, float& mean, float& m2, float cb,
                                           float mb, float m2b) {
  if (cb <= 0.f) return;
  const float tot = cnt + cb;
  const float delta = mb - mean;
  const float f = cb / tot;
  mean = fmaf(delta, f, mean);
  m2 = m2 + m2b + delta * delta * cnt * f;
  cnt = tot;
}

constexpr uint64_t kDrainTimeoutNs = 1000000000ull;

// Waits (bounded, ignoring the abort flag) until the most recent load into every stage of
// the ring has landed, so no TMA write into shared memory is in flight when the CTA exits.
// Load number q (0-based) went to stage q % stages as that stage's phase q / stages.
__device__ __forceinline__ void drain_loads(uint32_t bar_full, int stages, int issued) {
  for (int q = issued - 1; q >= 0 && q >= issued - stages; --q) {
    mbar_wait(bar_full + 8 * (q % stages), static_cast<uint32_t>((q / stages) & 1),
              kDrainTimeoutNs, nullptr);
  }
}

// Phase timestamps for latency studies, compiled out unless FO_PHASE_PROBE is defined:
// %globaltimer (ns) at entry (slots 0 and 8), setup done (1), first stage full at the MMA
// issuer (2), a unit's last MMA issued (3), its accumulator ready in the epilogue (4), all
// stores complete (5), exit (6 and 7).  Slots 3 and 4 hold the CTA's last unit.  One row
// of 16 per CTA.
#ifdef FO_PHASE_PROBE
static __device__ unsigned long long g_fo_probe[2048][16];
#define FO_PROBE(slot, v) (g_fo_probe[blockIdx.x & 2047][slot] = (v))
#else
#define FO_PROBE(slot, v) ((void)0)
#endif

template <int BN, int ACT, int OUT_DT, bool LN, bool CONV, bool PAIR, bool SWAP = false, int KPS = 1>
__global__ void __launch_bounds__(CONV ? 416 : 320, 1)
    fo_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmC, const KParams p) {
  constexpr int kProducerWarps = CONV ? 4 : 1;
  constexpr int kMmaWarp = kProducerWarps;
  constexpr int kFirstEpiWarp = kProducerWarps + 1;
  // PAIR: a cluster of two CTAs computes one 256 x BN tile with tcgen05 cta_group::2;
  // CTA r loads rows r*128.. of A and columns r*BN/2.. of B, holds rows r*128.. of the
  // accumulator in its TMEM and stores them.  The leader (rank 0) issues the MMAs.
  constexpr int kBHalf = PAIR ? BN / 2 : BN;  // B columns this CTA loads
  constexpr int kTileM = PAIR ? 2 * kBM : kBM;
  constexpr int kBStage = b_stage_bytes(kBHalf);
  static_assert(!PAIR || BN >= 128, "CTA pairs need BN >= 128");
  // SWAP (conv only): the MMA computes Y^T = W^T X^T, M = 128 output channels (A = weight
  // block, MN-major), N = BN output pixels (B = im2col tile, K-major), so a conv with few
  // channels still runs 128 x 256 MMAs; the epilogue transposes through shared memory.
  static_assert(!SWAP || (CONV && !PAIR && !LN), "operand swap is a single-CTA conv mode");
  constexpr int kOutBytes = OUT_DT == DT_F32 ? 4 : 2;
  constexpr int kCPC = 128 / kOutBytes;  // output columns per 128-byte chunk
  constexpr int kChunks = BN / kCPC;
  // Column halves of the epilogue: each half is taken by one warp of a lane quarter.  A
  // 16-bit BN 64 tile is a single 128-byte TMA store chunk; its two 32-column halves are
  // stored directly from registers instead (kNarrow: each lane writes its row's 64 bytes).
  constexpr bool kNarrow = !SWAP && kChunks == 1;
  constexpr int kHalves = 2;
  constexpr int kCW = kNarrow ? 32 : kCPC;                    // columns per epilogue step
  constexpr int kHalfChunks = kNarrow ? 1 : kChunks / kHalves;  // steps per half (non-swapped)
  constexpr int kHalfCols = BN / kHalves;                     // columns per half
  constexpr uint32_t kTmemCols = 2 * BN;
  static_assert(!LN || OUT_DT != DT_F32, "LayerNorm output is 16-bit");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int stages = p.stages;
  const uint32_t sA = smem_u32(smem);
  // KPS (k-blocks per stage) is a template parameter: the single MMA-issuing thread is
  // the bottleneck of this loop, and a runtime stage depth costs it measurable time
  constexpr int kps = KPS;
  static_assert(KPS == 1 || (KPS == 2 && !CONV), "two K slices per stage: GEMM family only");
  const uint32_t sB = sA + stages * kps * kAStageBytes;
  const uint32_t sEpi = sB + stages * kps * kBStage;
  uint8_t* misc = smem + (sEpi - sA) + epi_region_bytes(BN, PAIR ? 0 : p.csplit);
  // misc: [0,64) full[8] | [64,128) empty[8] | [128,144) tfull[2] | [144,160) tempty[2]
  //       | [160,168) drain | [168,176) red (cluster split) | [176,240) staged[8] (split
  //       partials, one per epilogue warp) | [248,256) tmem addr + abort flag
  //       | [256,320) lnld[8] (one-kernel LayerNorm: a stored slice read back, per warp)
  const uint32_t mb = smem_u32(misc);
  const uint32_t bar_full = mb;
  const uint32_t bar_empty = mb + 64;
  const uint32_t bar_tfull = mb + 128;
  const uint32_t bar_tempty = mb + 144;
  const uint32_t bar_drain = mb + 160;
  const uint32_t bar_red = mb + 168;  // cluster split: every partial this CTA receives has landed
  const uint32_t bar_staged = mb + 176;  // + 8 x epilogue warp: the other parts' partials are in smem
  const uint32_t bar_lnld = mb + 256;    // + 8 x epilogue warp: a stored LayerNorm slice is back in smem
  const int csplit = PAIR || CONV || LN ? 0 : p.csplit;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 248);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 252);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0;
  const int cid = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int ncl = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  if (threadIdx.x == 0) {
    FO_PROBE(0, global_timer_ns());
    FO_PROBE(8, global_timer_ns());
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(bar_full + 8 * s, (CONV && !p.conv_tma) ? 128 : 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_tfull + 8 * a, 1);
      mbar_init(bar_tempty + 8 * a, PAIR ? 2 * kEpiWarps : kEpiWarps);
    }
    mbar_init(bar_drain, 1);
    if (csplit > 1) mbar_init(bar_red, 1);
    for (int w = 0; w < kEpiWarps; ++w) mbar_init(bar_staged + 8 * w, 1);
    if (LN)
      for (int w = 0; w < kEpiWarps; ++w) mbar_init(bar_lnld + 8 * w, 1);
    *abort_flag = 0;
    fence_mbar_init();
    if (csplit > 1) {
      // Expect every byte the other parts will send: the chunks this CTA owns, once each.
      const int me = static_cast<int>(cluster_ctarank());
      const int cs = csplit > 1 ? csplit : 1;  // (a constant 0 in pair / conv / LayerNorm kernels)
      const int owned = (4 * (BN / 32) - me + cs - 1) / cs;
      mbar_arrive_expect_tx(bar_red, static_cast<uint32_t>((csplit - 1) * owned * 32 * 128));
    }
  }
  if (warp == kMmaWarp) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_slot), kTmemCols);
      tmem_relinquish();
    }
  }
  if (threadIdx.x == 32 * kFirstEpiWarp) {
    tma_prefetch_desc(&tmC);
    if (p.k_blocks > 0) {  // with K = 0 the A / B maps are left unencoded
      if (!CONV || p.conv_tma) tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
    }
  }
  // Every warp reconverges before a CTA-wide barrier: bar.sync counts a warp whose
  // lanes arrive at different times more than once, and would release the CTA early.
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before any remote use
  if (csplit > 1) cluster_sync();      // every receive barrier exists before any st.async
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint64_t tmo = p.timeout_ns;
  // Launched as a programmatic dependent of the previous kernel on the stream: the setup
  // above overlapped its tail; nothing below touches global memory before it completed.
  griddep_wait();
  if (threadIdx.x == 0) FO_PROBE(1, global_timer_ns());

  if (warp < kProducerWarps) {
    // ------------------------------------------------------------------ producer
    if constexpr (!CONV) {
      if (lane == 0) {
        int s = 0;
        uint32_t ph = 0;
        int issued = 0;  // stage loads issued by this thread
        bool ok = true;
        for (int u = cid; u < p.num_units && ok; u += ncl) {
          const Unit un = unit_of(p, u);
          const int tm = un.tm, tn = un.tn;
          for (int kb0 = un.kb0; kb0 < un.kb1; kb0 += kps) {
            const int nk = KPS == 1 ? 1 : min(KPS, un.kb1 - kb0);  // k-blocks in this stage
            if (!mbar_wait(bar_empty + 8 * s, ph ^ 1, tmo, abort_flag)) {
              ok = false;
              break;
            }
            const uint32_t fb = bar_full + 8 * s;
            const int arow = tm * kTileM + static_cast<int>(rank) * kBM;
            const int bcol = tn * BN + static_cast<int>(rank) * kBHalf;
            if constexpr (PAIR) {
              // Both CTAs' bytes complete on the leader's barrier; only the leader arrives.
              const uint32_t fbl = mapa_shared(fb, 0);
              if (rank == 0) mbar_arrive_expect_tx(fb, 2 * nk * (kAStageBytes + kBStage));
              for (int i = 0; i < nk; ++i) {
                const int kb = kb0 + i;
                const uint32_t sa = sA + (s * kps + i) * kAStageBytes, sb = sB + (s * kps + i) * kBStage;
                tma_load_2d_pair(sa, &tmA, fbl, kb * kBK, arow);
                if (p.b_mn) {
#pragma unroll
                  for (int j = 0; j < kBHalf / 64; ++j)
                    tma_load_2d_pair(sb + j * 64 * 128, &tmB, fbl, bcol + j * 64, kb * kBK);
                } else {
                  tma_load_2d_pair(sb, &tmB, fbl, kb * kBK, bcol);
                }
              }
            } else {
              mbar_arrive_expect_tx(fb, nk * (kAStageBytes + kBStage));
              for (int i = 0; i < nk; ++i) {
                const int kb = kb0 + i;
                const uint32_t sa = sA + (s * kps + i) * kAStageBytes, sb = sB + (s * kps + i) * kBStage;
                tma_load_2d(sa, &tmA, fb, kb * kBK, arow);
                if (p.b_mn) {
#pragma unroll
                  for (int j = 0; j < BN / 64; ++j)
                    tma_load_2d(sb + j * 64 * 128, &tmB, fb, bcol + j * 64, kb * kBK);
                } else {
                  tma_load_2d(sb, &tmB, fb, kb * kBK, bcol);
                }
              }
            }
            ++issued;
            if (++s == stages) {
              s = 0;
              ph ^= 1;
            }
          }
        }
        if (!ok) {
          record_error(p, kStatusTimeout, 0x10);
          *abort_flag = 1;
        }
        // A pair's loads complete on the leader's barriers: the leader drains both CTAs'
        // loads, and the closing cluster barrier keeps the peer alive until then.
        if (!PAIR || rank == 0) drain_loads(bar_full, stages, issued);
      }
    } else if (p.conv_tma) {
      // conv, TMA im2col: one thread loads each 128-pixel x 64-channel A tile of the
      // current filter tap with one instruction, and the weight tile beside it.
      if (threadIdx.x == 0) {
        int s = 0;
        uint32_t ph = 0;
        int issued = 0;
        bool ok = true;
        const int ohow = p.OH * p.OW;
        for (int u = cid; u < p.num_units && ok; u += ncl) {
          const Unit un = unit_of(p, u);
          const int tm = un.tm, tn = un.tn;
          const int m0 = SWAP ? tn * BN : tm * kTileM + static_cast<int>(rank) * kBM;
          const int n_img = m0 / ohow;
          const int rem = m0 - n_img * ohow;
          const int oh = rem / p.OW;
          const int ow = rem - oh * p.OW;
          const int w0 = ow * p.stride - p.pad;
          const int h0 = oh * p.stride - p.pad;
          for (int kb0 = un.kb0; kb0 < un.kb1; kb0 += kps) {
            const int nk = KPS == 1 ? 1 : min(KPS, un.kb1 - kb0);  // k-blocks in this stage
            if (!mbar_wait(bar_empty + 8 * s, ph ^ 1, tmo, abort_flag)) {
              ok = false;
              break;
            }
            const uint32_t fb = bar_full + 8 * s;
            const int bcol = tn * BN + static_cast<int>(rank) * kBHalf;
            if constexpr (PAIR) {
              if (rank == 0) mbar_arrive_expect_tx(fb, 2 * nk * (kAStageBytes + kBStage));
            } else {
              mbar_arrive_expect_tx(fb, nk * (kAStageBytes + kBStage));
            }
            for (int i = 0; i < nk; ++i) {
              const int kb = kb0 + i;
              const int tap = kb / p.c_blocks;
              const int cb = kb - tap * p.c_blocks;
              const int kh = tap / p.KW;
              const int kw = tap - kh * p.KW;
              const uint16_t ow16 = static_cast<uint16_t>(kw * p.dil), oh16 = static_cast<uint16_t>(kh * p.dil);
              const uint32_t sa = sA + (s * kps + i) * kAStageBytes, sb = sB + (s * kps + i) * kBStage;
              if constexpr (SWAP) {
#pragma unroll
                for (int j = 0; j < 2; ++j)  // A: 128 channels x 64 K of the weights, MN-major
                  tma_load_2d(sa + j * 64 * 128, &tmB, fb, tm * kBM + j * 64, tap * p.C + cb * kBK);
                tma_load_im2col_4d(sb, &tmA, fb, cb * kBK, w0, h0, n_img, ow16, oh16);  // B: BN pixels
              } else if constexpr (PAIR) {
                const uint32_t fbl = mapa_shared(fb, 0);
                tma_load_im2col_4d_pair(sa, &tmA, fbl, cb * kBK, w0, h0, n_img, ow16, oh16);
#pragma unroll
                for (int j = 0; j < kBHalf / 64; ++j)
                  tma_load_2d_pair(sb + j * 64 * 128, &tmB, fbl, bcol + j * 64, tap * p.C + cb * kBK);
              } else {
                tma_load_im2col_4d(sa, &tmA, fb, cb * kBK, w0, h0, n_img, ow16, oh16);
#pragma unroll
                for (int j = 0; j < BN / 64; ++j)
                  tma_load_2d(sb + j * 64 * 128, &tmB, fb, bcol + j * 64, tap * p.C + cb * kBK);
              }
            }
            ++issued;
            if (++s == stages) {
              s = 0;
              ph ^= 1;
            }
          }
        }
        if (!ok) {
          record_error(p, kStatusTimeout, 0x12);
          *abort_flag = 1;
        }
        // A pair's loads complete on the leader's barriers: the leader drains both CTAs'
        // loads, and the closing cluster barrier keeps the peer alive until then.
        if (!PAIR || rank == 0) drain_loads(bar_full, stages, issued);
      }
    } else {
      // conv gather: thread i of the warpgroup owns row i (one output pixel) of the A tile.
      const int i = threadIdx.x;  // 0..127
      constexpr int kLag = 2;
      int s = 0;
      uint32_t ph = 0;
      int issued = 0;  // cp.async groups committed by this thread
      bool ok = true;
      const int ohow = p.OH * p.OW;
      const char* xb = reinterpret_cast<const char*>(p.x);
      for (int u = cid; u < p.num_units && ok; u += ncl) {
        const Unit un = unit_of(p, u);
        const int tm = un.tm, tn = un.tn;
        const int m = tm * kBM + i;
        const bool valid_m = m < p.M;
        const int n_img = valid_m ? m / ohow : 0;
        const int rem = valid_m ? m - n_img * ohow : 0;
        const int oh = rem / p.OW;
        const int ow = rem - oh * p.OW;
        const int ih0 = oh * p.stride - p.pad;
        const int iw0 = ow * p.stride - p.pad;
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          const int tap = kb / p.c_blocks;
          const int cb = kb - tap * p.c_blocks;
          const int kh = tap / p.KW;
          const int kw = tap - kh * p.KW;
          if (!mbar_wait(bar_empty + 8 * s, ph ^ 1, tmo, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar_full + 8 * s;
          if (i == 0) {
            mbar_expect_tx(fb, kBStage);
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sB + s * kBStage + j * 64 * 128, &tmB, fb, tn * BN + j * 64,
                          tap * p.C + cb * kBK);
          }
          const int ih = ih0 + kh * p.dil;
          const int iw = iw0 + kw * p.dil;
          const bool inb = valid_m && ih >= 0 && ih < p.H && iw >= 0 && iw < p.W;
          const int c0 = cb * kBK;
          const char* src =
              xb + ((static_cast<long long>(n_img) * p.H + (inb ? ih : 0)) * p.W + (inb ? iw : 0)) *
                           static_cast<long long>(p.C) * 2 +
                       static_cast<long long>(c0) * 2;
          const uint32_t dst_row = sA + s * kAStageBytes + i * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const bool v = inb && (c0 + j * 8) < p.C;
            cp_async_16(dst_row + ((j ^ (i & 7)) << 4), v ? src + j * 16 : xb, v ? 16u : 0u);
          }
          cp_async_commit();
          ++issued;
          if (issued > kLag) {
            cp_async_wait<kLag>();
            fence_proxy_async_smem();
            int ss = s - kLag;
            if (ss < 0) ss += stages;
            mbar_arrive(bar_full + 8 * ss);
          }
          if (++s == stages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      cp_async_wait_all();
      fence_proxy_async_smem();
      // Arrive for the groups still owed (the last min(issued, kLag) stages).
      const int owed = issued < kLag ? issued : kLag;
      for (int j = owed; j >= 1; --j) {
        int ss = s - j;
        if (ss < 0) ss += stages;
        mbar_arrive(bar_full + 8 * ss);
      }
      if (!ok) {
        record_error(p, kStatusTimeout, 0x11);
        *abort_flag = 1;
      }
      if (i == 0) drain_loads(bar_full, stages, issued);  // the weight tiles
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      const int b_mn = SWAP ? 0 : p.b_mn;
      const uint32_t idesc = idesc_f16(p.ab_bf16, b_mn, BN, kTileM) | (SWAP ? (1u << 15) : 0u);  // [15]: A MN-major
      const uint64_t a_desc0 = SWAP ? sdesc_sw128(sA, 64 * 128, 1024) : sdesc_sw128(sA, 16, 1024);
      const uint32_t a_kstep = SWAP ? (2048 >> 4) : (32 >> 4);
      const uint64_t b_desc0 = b_mn ? sdesc_sw128(sB, 64 * 128, 1024) : sdesc_sw128(sB, 16, 1024);
      const uint32_t b_kstep = b_mn ? (2048 >> 4) : (32 >> 4);
      // One thread issues every MMA (~60 cycles each) and commit; the descriptors are
      // stepped per stage, not recomputed, and a pair frees a stage in both CTAs with one
      // commit, so the issue loop stays shorter than the MMAs it feeds.
      int s = 0;
      uint32_t ph = 0;
      uint64_t ad = a_desc0, bd = b_desc0;
      int acc = 0;
      uint32_t acc_ph = 0;
      bool ok = true;
      for (int u = cid; u < p.num_units && ok; u += ncl) {
        const Unit un = unit_of(p, u);
        const bool freed = PAIR ? mbar_wait_cluster(bar_tempty + 8 * acc, acc_ph ^ 1, tmo, abort_flag)
                                : mbar_wait(bar_tempty + 8 * acc, acc_ph ^ 1, tmo, abort_flag);
        if (!freed) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        uint32_t accum = 0;
        for (int kb0 = un.kb0; kb0 < un.kb1; kb0 += kps) {
          const int nk = KPS == 1 ? 1 : min(KPS, un.kb1 - kb0);
          if (!mbar_wait(bar_full + 8 * s, ph, tmo, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#ifdef FO_PHASE_PROBE
          if (u == cid && kb0 == un.kb0) FO_PROBE(2, global_timer_ns());
#endif
#pragma unroll 2
          for (int i = 0; i < nk; ++i) {
            const uint64_t a = ad + static_cast<uint64_t>(i * (kAStageBytes >> 4));
            const uint64_t b = bd + static_cast<uint64_t>(i * (kBStage >> 4));
            if constexpr (PAIR) {
              tc_mma_f16_pair(d, a, b, idesc, accum);
              tc_mma_f16_pair(d, a + a_kstep, b + b_kstep, idesc, 1u);
              tc_mma_f16_pair(d, a + 2 * a_kstep, b + 2 * b_kstep, idesc, 1u);
              tc_mma_f16_pair(d, a + 3 * a_kstep, b + 3 * b_kstep, idesc, 1u);
            } else {
              tc_mma_f16(d, a, b, idesc, accum);
              tc_mma_f16(d, a + a_kstep, b + b_kstep, idesc, 1u);
              tc_mma_f16(d, a + 2 * a_kstep, b + 2 * b_kstep, idesc, 1u);
              tc_mma_f16(d, a + 3 * a_kstep, b + 3 * b_kstep, idesc, 1u);
            }
            accum = 1u;
          }
          if constexpr (PAIR) {
            tc_commit_pair_both(bar_empty + 8 * s);  // free the stage in both CTAs
          } else {
            tc_commit(bar_empty + 8 * s);
          }
          if (++s == stages) {
            s = 0;
            ph ^= 1;
            ad = a_desc0;
            bd = b_desc0;
          } else {
            ad += static_cast<uint64_t>(kps * (kAStageBytes >> 4));
            bd += static_cast<uint64_t>(kps * (kBStage >> 4));
          }
        }
        if (!ok) break;
        FO_PROBE(3, global_timer_ns());
        if constexpr (PAIR) {  // both halves of the accumulator are ready
          tc_commit_pair_both(bar_tfull + 8 * acc);
        } else {
          tc_commit(bar_tfull + 8 * acc);
        }
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
      }
      if (!ok) {
        record_error(p, kStatusTimeout, 0x20);
        *abort_flag = 1;
      }
      // This CTA issues no more MMAs: a dependent row pass may begin launching (it waits
      // for the whole grid to finish before it reads any output).
      griddep_launch_dependents();
      // Drain: all issued MMAs complete before TMEM is released.
      if constexpr (PAIR) {
        tc_commit_pair(mapa_shared(bar_drain, 0));
      } else {
        tc_commit(bar_drain);
      }
      mbar_wait(bar_drain, 0, kDrainTimeoutNs, nullptr);
    }
  } else if (warp < kFirstEpiWarp + kEpiWarps) {
    // ------------------------------------------------------------------ epilogue
    const int ew = warp - kFirstEpiWarp;  // 0..7
    const int quarter = warp & 3;         // TMEM lane quarter this warp may access
    const int half = ew >> 2;             // column half of the tile this warp takes
    constexpr bool idle = false;           // every warp has a column half
    const int hcol = half * kHalfCols;    // first tile column of this warp's half
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t buf0 = sEpi + ew * kEpiBufBytes;
    int acc = 0;
    uint32_t acc_ph = 0;
    uint32_t nstore = 0;
    bool ok = true;
    // One-kernel LayerNorm (p.ln_fused): the slices this warp has stored centred and whose
    // statistics it has published, oldest first, normalised ln_defer units later.  A
    // row block's tiles lie within ln_span consecutive units, so after ln_defer =
    // ceil(ln_span / ncl) more units of this CTA every slice of the oldest one has been
    // published by some CTA's earlier (or same) unit, whose epilogue never waits on a later
    // unit: nothing can wait in a cycle.
    constexpr int kLnQ = kLnMaxDefer + 1;
    int h_tm[kLnQ] = {}, h_tn[kLnQ] = {};
    float h_sh[kLnQ] = {};
    int nh = 0;
    uint32_t ln_ph = 0;
    const int ln_defer = LN ? min(kLnMaxDefer, ln_defer_for(p.ln_span, ncl)) : 0;
    const uint32_t lnbar = bar_lnld + 8 * ew;
    // Normalises the slice (rows of this warp's lane quarter, columns of its half) of tile
    // (tm_, tn_) in place: waits until the last of the 2 x tiles_n slices of its 32 rows
    // has merged their statistics into (mean, rstd) (ln_cnt reaches 2 x tiles_n + 1),
    // reads the stored x - shift back through the staging block with TMA, writes
    // ((x - shift) + (shift - mean)) * rstd * gamma + beta and stores it.  `tail`: no
    // newer stores of this warp follow the slice's own, so wait for all of them.
    auto ln_normalize = [&](int tm_, int tn_, float sh_, bool tail) -> bool {
      const int r0 = tm_ * kTileM + static_cast<int>(rank) * kBM + quarter * 32;
      if (r0 >= p.M) return true;
      const int grp = r0 >> 5;
      const int target = 2 * p.tiles_n + 1;
      int ready = 1;
      if (lane == 0) {
        const int* cp = p.ln_cnt + grp;
        if (ld_acquire_gpu(cp) < target) {
          const uint64_t t0 = global_timer_ns();
          while (ld_acquire_gpu(cp) < target) {
            if (*abort_flag || global_timer_ns() - t0 > tmo) {
              ready = 0;
              break;
            }
            __nanosleep(64);
          }
        }
      }
      ready = __shfl_sync(0xffffffffu, ready, 0);
      __syncwarp();
      if (!ready) return false;
      // lane i holds row r0 + i's rstd and (shift - mean) * rstd
      const int row = r0 + lane;
      const float2 fin = row < p.M ? __ldcg(p.ln_fin + row) : make_float2(0.f, 0.f);
      const float rs = fin.y;
      const float ors = (sh_ - fin.x) * fin.y;
      if (lane == 0 && atomicAdd(p.ln_cnt + p.ln_groups + grp, 1) == target - 2) {
        // every normaliser of these rows has seen the arrivals: reset both counters
        atomicExch(p.ln_cnt + grp, 0);
        atomicExch(p.ln_cnt + p.ln_groups + grp, 0);
      }
#pragma unroll 1
      for (int ci = 0; ci < kHalfChunks; ++ci) {
        const int cbase = tn_ * BN + hcol + ci * kCW;
        // This lane's two columns of the 64-column chunk and their affine parameters,
        // loaded once for the chunk's 32 rows.
        const int col = cbase + 2 * lane;
        float g0 = 0.f, g1 = 0.f, b0 = 0.f, b1 = 0.f;
        if (col < p.N) {
          g0 = load_vec(p.gamma, p.vec_dtype, col);
          g1 = load_vec(p.gamma, p.vec_dtype, col + 1);
          b0 = load_vec(p.beta, p.vec_dtype, col);
          b1 = load_vec(p.beta, p.vec_dtype, col + 1);
        }
        if (lane == 0) {
          // the slice's stores have completed (only the newer stores of the current unit
          // may still be in flight) and the staging block is free
          if (tail) {
            bulk_wait<0>();
          } else {
            bulk_wait<kHalfChunks>();
            bulk_wait_read<0>();
          }
          fence_proxy_async_global();
          mbar_arrive_expect_tx(lnbar, kEpiBufBytes);
          tma_load_2d(buf0, &tmC, lnbar, cbase, r0);
        }
        if (!mbar_wait(lnbar, ln_ph, tmo, abort_flag)) return false;
        ln_ph ^= 1;
        // Row i of the staged 32 x 128 B block; this lane's 4 bytes sit in 16-byte chunk
        // lane / 4, swizzled by the row (32 lanes: 32 distinct banks).
#pragma unroll 8
        for (int i = 0; i < 32; ++i) {
          const float r = __shfl_sync(0xffffffffu, rs, i);
          const float o = __shfl_sync(0xffffffffu, ors, i);
          const uint32_t addr = buf0 + i * 128 + ((((lane >> 2) ^ (i & 7)) << 4) | ((lane & 3) << 2));
          uint32_t w;
          asm volatile("ld.shared.b32 %0, [%1];" : "=r"(w) : "r"(addr) : "memory");
          const float2 f = unpack2<OUT_DT>(w);
          // ((x - shift) + (shift - mean)) * rstd * gamma + beta
          w = pack2<OUT_DT>(fmaf(fmaf(f.x, r, o), g0, b0), fmaf(fmaf(f.y, r, o), g1, b1));
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(w) : "memory");
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // final values: written back first, before the slices still to be read back
          tma_store_2d_hint(&tmC, buf0, cbase, r0, l2_policy_evict_first());
          bulk_commit();
        }
        ++nstore;
      }
      return true;
    };
    // Normalises the oldest held slice and drops it from the queue.
    auto ln_pop = [&](bool tail) -> bool {
      const bool r = ln_normalize(h_tm[0], h_tn[0], h_sh[0], tail);
#pragma unroll
      for (int i = 0; i + 1 < kLnQ; ++i) {
        h_tm[i] = h_tm[i + 1];
        h_tn[i] = h_tn[i + 1];
        h_sh[i] = h_sh[i + 1];
      }
      --nh;
      return r;
    };
    // ln_fused == 2: the slice of tile (tm_, tn_) is still in accumulator acc_ (this warp's
    // rows and column half).  Waits for its 32 rows' merged (mean, rstd), then re-reads
    // TMEM, adds the bias (aff_: lane l holds column 32 j + l of the half), normalises and
    // stores each 64-column chunk once, and releases the accumulator.  Returns false when
    // the wait ran out (the accumulator is released all the same).
    auto ln_held = [&](int tm_, int tn_, int acc_, bool has_k_, const float2* aff_) -> bool {
      const int r0 = tm_ * kTileM + static_cast<int>(rank) * kBM + quarter * 32;
      bool good = true;
      float mean = 0.f, rstd = 0.f;
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR) {
            mbar_arrive_cluster(mapa_shared(bar_tempty + 8 * acc_, 0));
          } else {
            mbar_arrive(bar_tempty + 8 * acc_);
          }
        }
      };
      if (r0 >= p.M) {
        release();
        return true;
      }
      const int grp = r0 >> 5;
      const int target = 2 * p.tiles_n + 1;
      int ready = 1;
      if (lane == 0) {
        const int* cp = p.ln_cnt + grp;
        if (ld_acquire_gpu(cp) < target) {
          const uint64_t t0 = global_timer_ns();
          while (ld_acquire_gpu(cp) < target) {
            if (*abort_flag || global_timer_ns() - t0 > tmo) {
              ready = 0;
              break;
            }
            __nanosleep(64);
          }
        }
      }
      good = __shfl_sync(0xffffffffu, ready, 0) != 0;
      if (!good) {
        release();
        return false;
      }
      const int row = r0 + lane;  // lane i owns row r0 + i
      const float2 fin = row < p.M ? __ldcg(p.ln_fin + row) : make_float2(0.f, 0.f);
      mean = fin.x;
      rstd = fin.y;
      if (lane == 0 && atomicAdd(p.ln_cnt + p.ln_groups + grp, 1) == target - 2) {
        // every normaliser of these rows has seen the arrivals: reset both counters
        atomicExch(p.ln_cnt + grp, 0);
        atomicExch(p.ln_cnt + p.ln_groups + grp, 0);
      }
#pragma unroll 1
      for (int ci = 0; ci < kHalfChunks; ++ci) {
        const int tc = hcol + ci * kCW;
        const int cbase = tn_ * BN + tc;
        float v[kCW];
        {
          uint32_t q0[32], q1[32];
          tmem_ld_32x32b_x32(tmem_base + lane_off + acc_ * BN + tc, q0);
          if constexpr (kCW == 64) tmem_ld_32x32b_x32(tmem_base + lane_off + acc_ * BN + tc + 32, q1);
          tc_wait_ld_regs(q0);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = has_k_ ? __uint_as_float(q0[i]) : 0.f;
          if constexpr (kCW == 64) {
            tc_pin_regs(q1);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[32 + i] = has_k_ ? __uint_as_float(q1[i]) : 0.f;
          }
        }
        if (ci == kHalfChunks - 1) release();
        // lane l loads gamma / beta of column 32 h + l once; shuffles hand them out
#pragma unroll
        for (int h = 0; h < kCW / 32; ++h) {
          const int col = cbase + h * 32 + lane;
          const float gl = col < p.N ? load_vec(p.gamma, p.vec_dtype, col) : 0.f;
          const float bl = col < p.N ? load_vec(p.beta, p.vec_dtype, col) : 0.f;
          const float al = p.has_bias ? aff_[ci * (kCW / 32) + h].y : 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float x = v[h * 32 + i] + __shfl_sync(0xffffffffu, al, i);
            v[h * 32 + i] = fmaf((x - mean) * rstd, __shfl_sync(0xffffffffu, gl, i), __shfl_sync(0xffffffffu, bl, i));
          }
        }
        if (nstore >= 1) {
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
        }
        const uint32_t rowp = buf0 + lane * 128;
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const uint32_t w0 = pack2<OUT_DT>(v[8 * jj + 0], v[8 * jj + 1]);
          const uint32_t w1 = pack2<OUT_DT>(v[8 * jj + 2], v[8 * jj + 3]);
          const uint32_t w2 = pack2<OUT_DT>(v[8 * jj + 4], v[8 * jj + 5]);
          const uint32_t w3 = pack2<OUT_DT>(v[8 * jj + 6], v[8 * jj + 7]);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rowp + ((jj ^ (lane & 7)) << 4)), "r"(w0),
                       "r"(w1), "r"(w2), "r"(w3)
                       : "memory");
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d_hint(&tmC, buf0, cbase, r0, l2_policy_evict_first());
          bulk_commit();
        }
        ++nstore;
      }
      return true;
    };
    for (int u = cid; u < p.num_units; u += ncl) {
      const Unit un = unit_of(p, u);
      const int tm = un.tm, tn = un.tn;
      const bool has_k = un.kb1 > un.kb0;
      // The tile's per-column vectors (bias, or the BatchNorm affine) do not depend on
      // the accumulator: lane l loads columns hcol + 32 j + l before the wait, so their
      // latency overlaps the MMAs instead of following them.
      constexpr int kPre = SWAP ? 1 : kHalfCols / 32;
      float2 aff[kPre];
      if constexpr (!SWAP) {
        if (!idle) {
#pragma unroll
          for (int j = 0; j < kPre; ++j) aff[j] = channel_affine(p, tn * BN + hcol + j * 32 + lane);
        }
      }
      if (!mbar_wait(bar_tfull + 8 * acc, acc_ph, tmo, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (ew == 0 && lane == 0) FO_PROBE(4, global_timer_ns());
      if (idle) {
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR) {
            mbar_arrive_cluster(mapa_shared(bar_tempty + 8 * acc, 0));
          } else {
            mbar_arrive(bar_tempty + 8 * acc);
          }
        }
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
        continue;
      }
      if constexpr (!PAIR && !CONV && !LN) {
        if (csplit > 1) {
          // Cluster split.  This warp covers chunks gc = hcol/32 .. of its lane quarter;
          // chunk g = quarter * BN/32 + gc belongs to rank g % csplit.  First push the
          // partials of the chunks other ranks own into their receive areas, then reduce
          // the owned chunks (parts added in rank order: bitwise reproducible).
          const int me = static_cast<int>(cluster_ctarank());
          constexpr int kG = BN / 32;
          const int nown = csplit_owned_max(BN, csplit);
#pragma unroll
          for (int j = 0; j < kPre; ++j) {
            const int gc = hcol / 32 + j;
            const int g = quarter * kG + gc;
            const int owner = g % csplit;
            if (owner == me) continue;
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_base + lane_off + acc * BN + gc * 32, r);
            tc_wait_ld_regs(r);
            if (!has_k) {
#pragma unroll
              for (int i = 0; i < 32; ++i) r[i] = 0u;
            }
            const int slot = (me < owner ? me : me - 1) * nown + g / csplit;
            const uint32_t dst = mapa_shared(sEpi + slot * kRedChunkBytes + lane * kRedRowBytes, owner);
            const uint32_t rbar = mapa_shared(bar_red, owner);
#pragma unroll
            for (int i = 0; i < 8; ++i) st_async_v4(dst + 16 * i, r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3], rbar);
          }
          if (ew == 0 && lane == 0) FO_PROBE(12, global_timer_ns());
          bool landed = false;
          const int row = tm * kBM + quarter * 32 + lane;
#pragma unroll
          for (int j = 0; j < kPre; ++j) {
            const int gc = hcol / 32 + j;
            const int g = quarter * kG + gc;
            if (g % csplit != me) continue;
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_base + lane_off + acc * BN + gc * 32, r);
            tc_wait_ld_regs(r);
            if (!landed) {
              if (!mbar_wait_cluster(bar_red, 0, tmo, abort_flag)) {
                ok = false;
                break;
              }
              landed = true;
              if (lane == 0) FO_PROBE(13, global_timer_ns());
            }
            float t[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] = 0.f;
            for (int k = 0; k < csplit; ++k) {
              if (k == me) {
#pragma unroll
                for (int i = 0; i < 32; ++i) t[i] += has_k ? __uint_as_float(r[i]) : 0.f;
              } else {
                const int slot = (k < me ? k : k - 1) * nown + g / csplit;
                const float4* src = reinterpret_cast<const float4*>(smem + (sEpi - sA) + slot * kRedChunkBytes +
                                                                    lane * kRedRowBytes);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  const float4 q4 = src[i];
                  t[4 * i] += q4.x;
                  t[4 * i + 1] += q4.y;
                  t[4 * i + 2] += q4.z;
                  t[4 * i + 3] += q4.w;
                }
              }
            }
            if (p.has_bias) {
#pragma unroll
              for (int i = 0; i < 32; ++i) t[i] += __shfl_sync(0xffffffffu, aff[j].y, i);
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] = apply_act<ACT>(t[i]);
            const int cb = tn * BN + gc * 32;
            if (row < p.M) {
              char* dst = reinterpret_cast<char*>(p.out) + (static_cast<long long>(row) * p.ldo + cb) * kOutBytes;
              if (cb + 32 <= p.N) {
                if constexpr (OUT_DT == DT_F32) {
#pragma unroll
                  for (int i = 0; i < 8; ++i)
                    reinterpret_cast<float4*>(dst)[i] = make_float4(t[4 * i], t[4 * i + 1], t[4 * i + 2], t[4 * i + 3]);
                } else {
#pragma unroll
                  for (int i = 0; i < 4; ++i)
                    reinterpret_cast<uint4*>(dst)[i] =
                        make_uint4(pack2<OUT_DT>(t[8 * i], t[8 * i + 1]), pack2<OUT_DT>(t[8 * i + 2], t[8 * i + 3]),
                                   pack2<OUT_DT>(t[8 * i + 4], t[8 * i + 5]), pack2<OUT_DT>(t[8 * i + 6], t[8 * i + 7]));
                }
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                  if (cb + i >= p.N) continue;
                  if constexpr (OUT_DT == DT_F32) {
                    reinterpret_cast<float*>(dst)[i] = t[i];
                  } else {
                    reinterpret_cast<unsigned short*>(dst)[i] = static_cast<unsigned short>(pack2<OUT_DT>(t[i], 0.f) & 0xFFFFu);
                  }
                }
              }
            }
          }
          if (!ok) break;
          // Every TMEM load of this warp has completed: release the accumulator.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_tempty + 8 * acc);
          acc ^= 1;
          if (acc == 0) acc_ph ^= 1;
          continue;
        }
      }
      // Split tile: publish this part's fp32 partial of the warp's (quarter, half)
      // ([column][128 rows], coalesced), then the warp whose arrival completes that
      // (quarter, half) adds the other parts and runs the epilogue; the other warps
      // release the accumulator and move on.
      float* split_tile = nullptr;
      // Every part's partial of this warp's block (the own one included), in part order:
      // in shared memory when staged (kHalfCols x 32 floats apart), else in the workspace
      // (8 blocks apart).  The sum is taken over these in part order, so a split tile is
      // bitwise reproducible whichever part arrives last.
      const float* parts_base = nullptr;
      bool staged = false;
      constexpr int kRegionFloats = kHalfCols * 32;  // one (part, quarter, half) block
      // split slot of this CTA's 128 rows (a CTA pair's tile has two)
      const int sti = PAIR ? un.st * 2 + static_cast<int>(rank) : un.st;
      if (un.st >= 0) {
        split_tile = p.split_ws + static_cast<long long>(sti) * p.split * BN * 128;
        float* mine = split_tile + static_cast<long long>((un.part * 4 + quarter) * 2 + half) * kRegionFloats + lane;
#pragma unroll 1
        for (int c = 0; c < kHalfCols / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + lane_off + acc * BN + hcol + c * 32, r);
          tc_wait_ld_regs(r);
#pragma unroll
          for (int i = 0; i < 32; ++i) __stcg(mine + (c * 32 + i) * 32, __uint_as_float(r[i]));
        }
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(p.split_cnt + sti * 8 + quarter * 2 + half, 1) == p.split - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR) {
              mbar_arrive_cluster(mapa_shared(bar_tempty + 8 * acc, 0));
            } else {
              mbar_arrive(bar_tempty + 8 * acc);
            }
          }
          acc ^= 1;
          if (acc == 0) acc_ph ^= 1;
          continue;
        }
        __threadfence();
        if (lane == 0) p.split_cnt[sti * 8 + quarter * 2 + half] = 0;
        // On the CTA's last unit (automatic plans give every split unit its own CTA, after
        // all whole tiles) whose MMAs are complete, the pipeline ring is idle: each
        // epilogue warp copies the other parts' blocks into its share of it with one bulk
        // copy per part (deep in flight, where loads into registers kept ~4 KB per warp in
        // flight and ran at ~30 GB/s per SM).  At most once per CTA, so its barrier runs
        // one phase.
        const int ring_share = (p.stages * kps * (kAStageBytes + kBStage) / kEpiWarps) & ~15;
        // Two parts: own + other is one addition, the same bits in either order, so only the
        // other part's block is staged (a 256-column half's 16 KB fits a warp's share).
        const bool two = p.split == 2;
        const uint32_t need = static_cast<uint32_t>((two ? 1 : p.split) * kRegionFloats * 4);
        staged = static_cast<int>(need) <= ring_share && u + ncl >= p.num_units;
        const uint32_t dst = sA + ew * ring_share;
        const uint32_t wbar = bar_staged + 8 * ew;
        if (staged) {
          if (lane == 0) {
            fence_proxy_async_global();  // the parts' generic stores, seen by the bulk copies
            mbar_arrive_expect_tx(wbar, need);
            for (int q = 0; q < p.split; ++q) {
              if (two && q == un.part) continue;
              bulk_load_g2s(dst + (two ? 0 : q) * kRegionFloats * 4,
                            split_tile + static_cast<long long>((q * 4 + quarter) * 2 + half) * kRegionFloats,
                            kRegionFloats * 4, wbar);
            }
          }
          // one phase per kernel: a CTA runs at most one split unit
          if (!mbar_wait(wbar, 0, tmo, abort_flag)) {
            ok = false;
            break;
          }
          parts_base = reinterpret_cast<const float*>(smem + (dst - sA)) + lane;
        } else {
          parts_base = split_tile + static_cast<long long>((quarter * 2 + half) * kRegionFloats) + lane;
        }
      }
      // Column `col` (within the half) of part q of this warp's block.
      auto part_value = [&](int q, int col) -> float {
        if (staged) return parts_base[(q * kHalfCols + col) * 32];
        return __ldcg(parts_base + static_cast<long long>(q) * 8 * kRegionFloats + col * 32);
      };
      // Two parts: column `col` of the other part's block.
      auto other_value = [&](int col) -> float {
        if (staged) return parts_base[col * 32];
        return __ldcg(parts_base + static_cast<long long>(1 - un.part) * 8 * kRegionFloats + col * 32);
      };
      float st_cnt = 0.f, st_mean = 0.f, st_m2 = 0.f;
      float shift = 0.f;  // LayerNorm: the tile is stored centred on its first chunk's mean
      if constexpr (SWAP) {
        // TMEM lane = output channel f, column = output pixel.  Each 32-pixel chunk is
        // transposed through shared memory ([pixel][32 channels], unswizzled) and stored
        // as a 32 x 32 block of the NHWC output.  The warp's 4 KB of staging holds
        // kSwapBufs such blocks, so that many TMA stores stay in flight.  The warp takes
        // the chunks of its column half (pixels hcol .. hcol + BN/2 of the tile).
        const int f = tm * kBM + quarter * 32 + lane;
        const int f0 = tm * kBM + quarter * 32;
        const float2 aff = channel_affine(p, f);
        constexpr int kRowB = 32 * kOutBytes;
        constexpr int kSwapBox = 32 * kRowB;
        constexpr int kSwapBufs = kEpiBufBytes / kSwapBox;
        constexpr int kC0 = 0, kCn = kHalfCols / 32;  // chunks of a half
        const int cfirst = hcol / 32;
        // Residual of the BN-add-ReLU epilogue.  Whole 32-channel groups: each lane loads
        // one pixel's 32 channels (4 x 16 B) one chunk ahead, and the chunk is transposed
        // through the staging block it will be stored from.  A partial channel group
        // (F not a multiple of 32) reads element by element.
        const bool vec_add = OUT_DT != DT_F32 && p.add_src != nullptr && f0 + 32 <= p.N;
        const unsigned short* add_col = OUT_DT != DT_F32 && p.add_src != nullptr && !vec_add && f < p.N
                                            ? reinterpret_cast<const unsigned short*>(p.add_src) + f
                                            : nullptr;
        const unsigned short* add_grp = vec_add ? reinterpret_cast<const unsigned short*>(p.add_src) + f0 : nullptr;
        uint4 qn[4] = {};
        auto load_res = [&](int c) {
          const int px = tn * BN + c * 32 + lane;
          if (px < p.M) {
            const uint4* src = reinterpret_cast<const uint4*>(add_grp + static_cast<long long>(px) * p.ld_add);
#pragma unroll
            for (int j = 0; j < 4; ++j) qn[j] = __ldg(src + j);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) qn[j] = make_uint4(0u, 0u, 0u, 0u);
          }
        };
        if (vec_add) load_res(cfirst);
#pragma unroll 1
        for (int ci = kC0; ci < kCn; ++ci) {
          const int c = cfirst + ci;
          uint4 q[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) q[j] = qn[j];
          if (vec_add && ci + 1 < kCn) load_res(c + 1);
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + lane_off + acc * BN + c * 32, r);
          tc_wait_ld_regs(r);
          if (ci == kCn - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_tempty + 8 * acc);
          }
          const uint32_t buf = buf0 + (nstore % kSwapBufs) * kSwapBox;
          if (nstore >= kSwapBufs) {
            if (lane == 0) bulk_wait_read<kSwapBufs - 1>();
            __syncwarp();
          }
          float acc_v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) acc_v[i] = has_k ? __uint_as_float(r[i]) : 0.f;
          if (split_tile != nullptr && p.split == 2) {  // own + other: either order, same bits
#pragma unroll
            for (int i = 0; i < 32; ++i) acc_v[i] += other_value(c * 32 - hcol + i);
          } else if (split_tile != nullptr) {  // every part, in part order (reproducible)
#pragma unroll
            for (int i = 0; i < 32; ++i) acc_v[i] = 0.f;
            for (int qq = 0; qq < p.split; ++qq) {
#pragma unroll
              for (int i = 0; i < 32; ++i) acc_v[i] += part_value(qq, c * 32 - hcol + i);
            }
          }
          if (p.bn_mode) {
#pragma unroll
            for (int i = 0; i < 32; ++i) acc_v[i] = fmaf(round_in(acc_v[i], p.ab_bf16), aff.x, aff.y);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) acc_v[i] = fmaf(acc_v[i], aff.x, aff.y);
          }
          if constexpr (OUT_DT != DT_F32) {
            if (vec_add) {
              // pixel rows in, channel columns out: every lane reads back exactly the
              // elements it overwrites below, so one warp barrier suffices
#pragma unroll
              for (int j = 0; j < 4; ++j)
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(buf + lane * kRowB + j * 16),
                             "r"(q[j].x), "r"(q[j].y), "r"(q[j].z), "r"(q[j].w)
                             : "memory");
              __syncwarp();
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                unsigned short h;
                asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(buf + i * kRowB + lane * 2) : "memory");
                acc_v[i] += unpack2<OUT_DT>(static_cast<uint32_t>(h)).x;
              }
            } else if (add_col != nullptr) {
              const int px0 = tn * BN + c * 32;
#pragma unroll
              for (int i = 0; i < 32; ++i)
                acc_v[i] += px0 + i < p.M ? load_vec(add_col + static_cast<long long>(px0 + i) * p.ld_add, OUT_DT, 0)
                                          : 0.f;
            }
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float val = apply_act<ACT>(acc_v[i]);
            const uint32_t addr = buf + i * kRowB + lane * kOutBytes;
            if constexpr (OUT_DT == DT_F32) {
              asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(__float_as_uint(val)) : "memory");
            } else {
              const unsigned short h = static_cast<unsigned short>(pack2<OUT_DT>(val, 0.f) & 0xFFFFu);
              asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(h) : "memory");
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, buf, tm * kBM + quarter * 32, tn * BN + c * 32);
            bulk_commit();
          }
          ++nstore;
        }
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
        continue;
      }
      const int row0 = tm * kTileM + static_cast<int>(rank) * kBM + quarter * 32;
      const int col0 = tn * BN;
#pragma unroll
      for (int ci = 0; ci < kHalfChunks; ++ci) {
        const int tc = hcol + ci * kCW;  // first tile column of this step
        const int cbase = col0 + tc;
        float v[kCW];
        {
          // Both 32-column loads of a 64-column step are in flight before one wait.
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(tmem_base + lane_off + acc * BN + tc, r0);
          if constexpr (kCW == 64) tmem_ld_32x32b_x32(tmem_base + lane_off + acc * BN + tc + 32, r1);
          tc_wait_ld_regs(r0);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = has_k ? __uint_as_float(r0[i]) : 0.f;
          if constexpr (kCW == 64) {
            tc_pin_regs(r1);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[32 + i] = has_k ? __uint_as_float(r1[i]) : 0.f;
          }
        }
        if (split_tile != nullptr && p.split == 2) {  // own + other: either order, same bits
#pragma unroll
          for (int i = 0; i < kCW; ++i) v[i] += other_value(tc - hcol + i);
        } else if (split_tile != nullptr) {  // every part, in part order (reproducible)
#pragma unroll
          for (int i = 0; i < kCW; ++i) v[i] = 0.f;
          for (int q = 0; q < p.split; ++q) {
#pragma unroll
            for (int i = 0; i < kCW; ++i) v[i] += part_value(q, tc - hcol + i);
          }
        }
        if (ci == kHalfChunks - 1 && !(LN && p.ln_fused == 2)) {
          // The accumulator buffer is free once every lane's loads of it have completed.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR) {
              mbar_arrive_cluster(mapa_shared(bar_tempty + 8 * acc, 0));
            } else {
              mbar_arrive(bar_tempty + 8 * acc);
            }
          }
        }
        if (p.bn_mode) {  // lane i holds column i's folded BatchNorm; shuffles broadcast it
#pragma unroll
          for (int h = 0; h < kCW / 32; ++h) {
            const float2 a2 = aff[ci * (kCW / 32) + h];
#pragma unroll
            for (int i = 0; i < 32; ++i)
              v[h * 32 + i] = fmaf(round_in(v[h * 32 + i], p.ab_bf16), __shfl_sync(0xffffffffu, a2.x, i),
                                   __shfl_sync(0xffffffffu, a2.y, i));
          }
        } else if (p.has_bias) {
#pragma unroll
          for (int h = 0; h < kCW / 32; ++h) {
            const float bl = aff[ci * (kCW / 32) + h].y;
#pragma unroll
            for (int i = 0; i < 32; ++i) v[h * 32 + i] += __shfl_sync(0xffffffffu, bl, i);
          }
        }
        if constexpr (CONV && OUT_DT != DT_F32) {
          // residual of the BN-add-ReLU epilogue: this lane's output row, kCW columns
          const int row = row0 + lane;
          if (p.add_src != nullptr && row < p.M) {
            const unsigned short* ar = reinterpret_cast<const unsigned short*>(p.add_src) + row * p.ld_add + cbase;
            if (cbase + kCW <= p.N) {
#pragma unroll
              for (int j = 0; j < kCW / 8; ++j) {
                const uint4 q = __ldg(reinterpret_cast<const uint4*>(ar) + j);
                const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 f2 = unpack2<OUT_DT>(w[e]);
                  v[8 * j + 2 * e] += f2.x;
                  v[8 * j + 2 * e + 1] += f2.y;
                }
              }
            } else {
#pragma unroll
              for (int i = 0; i < kCW; ++i)
                if (cbase + i < p.N) v[i] += load_vec(ar, OUT_DT, i);
            }
          }
        }
#pragma unroll
        for (int i = 0; i < kCW; ++i) v[i] = apply_act<ACT>(v[i]);
        if constexpr (LN) {
          // Shifted sums: shift = the row's first value of this slice (a sample of the
          // row, so |mean - shift| is of the order of the row's spread), d = x - shift,
          // S1 = sum d, S2 = sum d^2; the slice's (mean, M2) = (shift + S1 / n,
          // S2 - S1^2 / n).  d is also what is stored: the 16-bit rounding then scales
          // with the row's spread, not with its mean; the normaliser adds
          // (shift - row mean) back in fp32.
          if (ci == 0) shift = v[0];
          const int cv = min(kCW, p.N - cbase);
          float s1[4] = {0.f, 0.f, 0.f, 0.f}, s2[4] = {0.f, 0.f, 0.f, 0.f};
          if (cv >= kCW) {
#pragma unroll
            for (int i = 0; i < kCW; ++i) {
              const float d = v[i] - shift;
              s1[i & 3] += d;
              s2[i & 3] = fmaf(d, d, s2[i & 3]);
              v[i] = d;
            }
          } else {
#pragma unroll
            for (int i = 0; i < kCW; ++i) {
              const float d = i < cv ? v[i] - shift : 0.f;
              s1[i & 3] += d;
              s2[i & 3] = fmaf(d, d, s2[i & 3]);
              v[i] = d;
            }
          }
          st_cnt += static_cast<float>(max(cv, 0));
          st_mean += (s1[0] + s1[1]) + (s1[2] + s1[3]);  // S1 until the slice ends
          st_m2 += (s2[0] + s2[1]) + (s2[2] + s2[3]);    // S2 until the slice ends
        }
        if (LN && p.ln_fused == 2) {
          // held in TMEM: stored once, normalised, by ln_held below
        } else if constexpr (kNarrow) {
          // 16-bit BN 64: lane l stores row row0 + l of this 32-column half, 64
          // contiguous bytes, straight from registers.
          const int row = row0 + lane;
          if (row < p.M) {
            unsigned short* dst = reinterpret_cast<unsigned short*>(p.out) + static_cast<long long>(row) * p.ldo + cbase;
            if (cbase + 32 <= p.N) {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                reinterpret_cast<uint4*>(dst)[j] =
                    make_uint4(pack2<OUT_DT>(v[8 * j + 0], v[8 * j + 1]), pack2<OUT_DT>(v[8 * j + 2], v[8 * j + 3]),
                               pack2<OUT_DT>(v[8 * j + 4], v[8 * j + 5]), pack2<OUT_DT>(v[8 * j + 6], v[8 * j + 7]));
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (cbase + i < p.N) dst[i] = static_cast<unsigned short>(pack2<OUT_DT>(v[i], 0.f) & 0xFFFFu);
            }
          }
        } else {
          // Stage the 32 x 128 B block in swizzled shared memory, then TMA-store it.
          const uint32_t buf = buf0;
          if (nstore >= 1) {
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
          }
          const uint32_t rowp = buf + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint32_t w0, w1, w2, w3;
            if constexpr (OUT_DT == DT_F32) {
              w0 = __float_as_uint(v[4 * j + 0]);
              w1 = __float_as_uint(v[4 * j + 1]);
              w2 = __float_as_uint(v[4 * j + 2]);
              w3 = __float_as_uint(v[4 * j + 3]);
            } else {
              w0 = pack2<OUT_DT>(v[8 * j + 0], v[8 * j + 1]);
              w1 = pack2<OUT_DT>(v[8 * j + 2], v[8 * j + 3]);
              w2 = pack2<OUT_DT>(v[8 * j + 4], v[8 * j + 5]);
              w3 = pack2<OUT_DT>(v[8 * j + 6], v[8 * j + 7]);
            }
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rowp + ((j ^ (lane & 7)) << 4)),
                         "r"(w0), "r"(w1), "r"(w2), "r"(w3)
                         : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (LN && p.ln_fused) {
              // the centred slice is read back a unit later: keep it in L2
              tma_store_2d_hint(&tmC, buf, cbase, row0, l2_policy_evict_last());
            } else {
              tma_store_2d(&tmC, buf, cbase, row0);
            }
            bulk_commit();
          }
          ++nstore;
        }
      }
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1;

      if constexpr (LN) {
        const int row = row0 + lane;
        // (S1, S2) of the slice's shifted values -> (mean, M2)
        if (st_cnt > 0.f) {
          const float s1 = st_mean;
          st_mean = shift + s1 / st_cnt;
          st_m2 = fmaxf(0.f, st_m2 - s1 * (s1 / st_cnt));
        } else {
          st_mean = st_m2 = 0.f;
        }
        if (!kNarrow && p.ln_fused) {
          // Publish this slice's (mean, M2), count it into its 32 rows' arrivals, hold
          // it, and normalise the oldest held slice once ln_defer newer ones exist.
          if (row < p.M)
            p.ln_st2[static_cast<long long>(tn * kHalves + half) * p.M + row] = make_float2(st_mean, st_m2);
          __threadfence();
          __syncwarp();
          if (row0 < p.M) {
            // The warp whose arrival completes its 32 rows merges their 2 x tiles_n slices
            // once (slice order, Chan et al.), publishes (mean, rstd) per row and counts
            // once more: normalisers wait for 2 x tiles_n + 1.
            const int nsl = 2 * p.tiles_n;
            int last = 0;
            if (lane == 0) last = atomicAdd(p.ln_cnt + (row0 >> 5), 1) == nsl - 1;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
              __threadfence();
              float c = 0.f, mean = 0.f, m2 = 0.f;
              if (row < p.M) {
                for (int s0 = 0; s0 < nsl; s0 += 8) {
                  float2 v[8];
#pragma unroll
                  for (int i = 0; i < 8; ++i)
                    v[i] = s0 + i < nsl ? __ldcg(p.ln_st2 + static_cast<long long>(s0 + i) * p.M + row)
                                        : make_float2(0.f, 0.f);
#pragma unroll
                  for (int i = 0; i < 8; ++i)
                    chan_merge(c, mean, m2, static_cast<float>(max(0, min(kHalfCols, p.N - (s0 + i) * kHalfCols))),
                               v[i].x, v[i].y);
                }
                p.ln_fin[row] = make_float2(mean, rsqrtf(m2 / static_cast<float>(p.N) + p.eps));
              }
              __threadfence();
              __syncwarp();
              if (lane == 0) red_add_release_gpu(p.ln_cnt + (row0 >> 5), 1);
            }
          }
          if (p.ln_fused == 2) {
            // the accumulator just flipped: this unit's slice is in buffer acc ^ 1
            if (!ln_held(tm, tn, acc ^ 1, has_k, aff)) {
              ok = false;
              break;
            }
          } else {
#pragma unroll
            for (int i = 0; i < kLnQ; ++i) {
              if (i == nh) {
                h_tm[i] = tm;
                h_tn[i] = tn;
                h_sh[i] = shift;
              }
            }
            ++nh;
            if (nh > ln_defer && !ln_pop(false)) {
              ok = false;
              break;
            }
          }
        } else {
          // Per-tile row statistics; the row pass (launched next on the same stream)
          // merges them and normalises every row in place.  The slice is this warp's
          // column half of the tile.
          if (row < p.M)
            p.ln_stats[static_cast<long long>(tn * kHalves + half) * p.M + row] = make_float4(st_mean, st_m2, shift, 0.f);
        }
      }
    }
    if constexpr (LN) {
      // the slices still held after the last unit
      while (ok && nh > 0) {
        if (!ln_pop(true)) ok = false;
      }
    }
    if (!ok) {
      record_error(p, kStatusTimeout, 0x30);
      *abort_flag = 1;
    }
    // Only the staging buffers' reads must finish before the CTA exits; the stores
    // themselves complete with the grid, before any later kernel on the stream runs.
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
    if (ew == 0 && lane == 0) FO_PROBE(5, global_timer_ns());
  }

  __syncwarp();  // the producer and MMA warps ran their loops on lane 0 alone
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // no CTA leaves while its peer may still use it
  if (csplit > 1) cluster_sync();
  if (threadIdx.x == 0) {
    FO_PROBE(6, global_timer_ns());
    FO_PROBE(7, global_timer_ns());
  }
  if (threadIdx.x == 5) FO_PROBE(9, global_timer_ns());
  if (threadIdx.x == 32 * kMmaWarp) FO_PROBE(10, global_timer_ns());
  if (threadIdx.x == 32 * kFirstEpiWarp) FO_PROBE(11, global_timer_ns());
  if (warp == kMmaWarp) {
    tc_fence_after();
    if constexpr (PAIR) {
      tmem_dealloc_pair(tmem_base, kTmemCols);
    } else {
      tmem_dealloc(tmem_base, kTmemCols);
    }
  }
}

// Eight consecutive elements of a parameter vector (16-byte aligned start) as floats.

// Second pass of the fused LayerNorm: one warp per output row.  The lanes merge the
// row's tiles_n slice statistics (Chan et al.) into mean / rstd with a butterfly of
// shuffles, then normalise the row in place: y = (x_stored + shift - mean) * rstd *
// gamma + beta, where shift is the value the GEMM epilogue subtracted before storing
// that slice.  Each lane keeps 8 x 16-byte loads in flight.  Grid-wide and
// stream-ordered after the GEMM kernel, so it runs at full-chip bandwidth on rows that
// are mostly still in L2.
template <int OUT_DT>
__global__ void __launch_bounds__(256) fo_ln_normalize_kernel(const KParams p, int bn) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  griddep_wait();
  if (row >= p.M) return;
  unsigned short* rowp = reinterpret_cast<unsigned short*>(p.out) + static_cast<long long>(row) * p.ldo;
  const int slabs = (p.N + 255) / 256;
  for (int s0 = 0; s0 < slabs; s0 += 8) {
    // Issue this batch's row loads first so they overlap the statistics merge.
    uint4 y[8];
    float sh[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int col = (s0 + u) * 256 + lane * 8;
      if (s0 + u < slabs && col < p.N) {
        y[u] = __ldcg(reinterpret_cast<const uint4*>(rowp + col));
        sh[u] = __ldcg(p.ln_stats + static_cast<long long>(col / bn) * p.M + row).z;
      }
    }
    float cnt = 0.f, mean = 0.f, m2 = 0.f;
    for (int j = lane; j < p.tiles_n; j += 32) {
      const float4 pm = __ldcg(p.ln_stats + static_cast<long long>(j) * p.M + row);
      chan_merge(cnt, mean, m2, static_cast<float>(min(bn, p.N - j * bn)), pm.x, pm.y);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float c2 = __shfl_xor_sync(0xffffffffu, cnt, o);
      const float m2b = __shfl_xor_sync(0xffffffffu, m2, o);
      const float mb = __shfl_xor_sync(0xffffffffu, mean, o);
      chan_merge(cnt, mean, m2, c2, mb, m2b);
    }
    const float rs = rsqrtf(m2 / static_cast<float>(p.N) + p.eps);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int col = (s0 + u) * 256 + lane * 8;
      if (s0 + u < slabs && col < p.N) {
        const float off = sh[u] - mean;
        float g[8], b[8];
        load_vec8(p.gamma, p.vec_dtype, col, g);
        load_vec8(p.beta, p.vec_dtype, col, b);
        uint32_t w[4] = {y[u].x, y[u].y, y[u].z, y[u].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack2<OUT_DT>(w[e]);
          w[e] = pack2<OUT_DT>(fmaf((f.x + off) * rs, g[2 * e], b[2 * e]),
                               fmaf((f.y + off) * rs, g[2 * e + 1], b[2 * e + 1]));
        }
        __stcg(reinterpret_cast<uint4*>(rowp + col), make_uint4(w[0], w[1], w[2], w[3]));
      }
    }
  }
}

// Row pass of both LayerNorm epilogues for N <= 1024 * kChunks: one 128-thread block per
// row, each thread owning kChunks 8-element groups (columns chunk * 1024 + tid * 8), so
// every load of the row is issued at once and the pass costs about one memory round trip
// plus two block reductions.  gamma, beta and the residual do not depend on the GEMM and
// are read before griddep_wait(), overlapping the GEMM's tail when the launch is
// programmatic.
//   RESID false (FO_EPI_BIAS_LN): the stored row is centred per BN slice; the slices'
//     (mean, M2, shift) statistics are merged (Chan et al.) into the row's mean / rstd.
//   RESID true (FO_EPI_BIAS_RESIDUAL_LN): x = stored (A.B + bias, rounded) + residual,
//     rounded to the 16-bit output type as the reference's fp16 tensor add does; mean
//     and variance are two-pass block reductions over the registers.
// Its registers limit it to ~4 blocks per SM, so it is the small-M pass (every row of a
// small problem resident at once); large M goes to the warp-per-row kernels.
template <int OUT_DT, bool RESID, int kChunks>
__global__ void __launch_bounds__(128) fo_ln_rows_kernel(const KParams p, int bn) {
  __shared__ float red[3][4];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long row = blockIdx.x;
  unsigned short* rowp = reinterpret_cast<unsigned short*>(p.out) + row * p.ldo;
  float g[kChunks][8], b[kChunks][8];
  uint4 r[RESID ? kChunks : 1];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = c * 1024 + tid * 8;
    if (col < p.N) {
      load_vec8(p.gamma, p.vec_dtype, col, g[c]);
      load_vec8(p.beta, p.vec_dtype, col, b[c]);
      if constexpr (RESID)
        r[c] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned short*>(p.residual) +
                                                   row * p.ldr + col));
    }
  }
  griddep_wait();
  uint4 y[kChunks];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = c * 1024 + tid * 8;
    if (col < p.N) y[c] = __ldcg(reinterpret_cast<const uint4*>(rowp + col));
  }
  // x values of chunk c, in fp32
  auto xval = [&](int c, float (&x)[8]) {
    const uint32_t wy[4] = {y[c].x, y[c].y, y[c].z, y[c].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = unpack2<OUT_DT>(wy[e]);
      x[2 * e] = a.x;
      x[2 * e + 1] = a.y;
    }
    if constexpr (RESID) {  // x = round16(y + residual), the reference's 16-bit add
      const uint32_t wr[4] = {r[c].x, r[c].y, r[c].z, r[c].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a = unpack2<OUT_DT>(wr[e]);
        const float2 q = unpack2<OUT_DT>(pack2<OUT_DT>(x[2 * e] + a.x, x[2 * e + 1] + a.y));
        x[2 * e] = q.x;
        x[2 * e + 1] = q.y;
      }
    }
  };
  float mean, rs;
  float sh[kChunks];  // per-chunk shift to add back (LN: slice shift - mean; residual: -mean)
  if constexpr (RESID) {
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      if (c * 1024 + tid * 8 < p.N) {
        float x[8];
        xval(c, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) sum += x[e];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[0][warp] = sum;
    __syncthreads();
    mean = (red[0][0] + red[0][1] + red[0][2] + red[0][3]) / static_cast<float>(p.N);
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      if (c * 1024 + tid * 8 < p.N) {
        float x[8];
        xval(c, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) q += (x[e] - mean) * (x[e] - mean);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    if (lane == 0) red[1][warp] = q;
    __syncthreads();
    rs = rsqrtf((red[1][0] + red[1][1] + red[1][2] + red[1][3]) / static_cast<float>(p.N) + p.eps);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) sh[c] = -mean;
  } else {
    // slice statistics: thread j < tiles_n reads slice j's; each chunk's shift
    float cnt = 0.f, m = 0.f, m2 = 0.f;
    for (int j = tid; j < p.tiles_n; j += 128) {
      const float4 pm = __ldcg(p.ln_stats + static_cast<long long>(j) * p.M + row);
      chan_merge(cnt, m, m2, static_cast<float>(min(bn, p.N - j * bn)), pm.x, pm.y);
    }
    float shift[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const int col = c * 1024 + tid * 8;
      shift[c] = col < p.N ? __ldcg(p.ln_stats + static_cast<long long>(col / bn) * p.M + row).z : 0.f;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float c2 = __shfl_xor_sync(0xffffffffu, cnt, o);
      const float mb = __shfl_xor_sync(0xffffffffu, m, o);
      const float m2b = __shfl_xor_sync(0xffffffffu, m2, o);
      chan_merge(cnt, m, m2, c2, mb, m2b);
    }
    if (lane == 0) {
      red[0][warp] = cnt;
      red[1][warp] = m;
      red[2][warp] = m2;
    }
    __syncthreads();
    cnt = red[0][0];
    m = red[1][0];
    m2 = red[2][0];
#pragma unroll
    for (int w = 1; w < 4; ++w) chan_merge(cnt, m, m2, red[0][w], red[1][w], red[2][w]);
    mean = m;
    rs = rsqrtf(m2 / static_cast<float>(p.N) + p.eps);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) sh[c] = shift[c] - mean;
  }
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = c * 1024 + tid * 8;
    if (col < p.N) {
      float x[8];
      xval(c, x);
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        w[e] = pack2<OUT_DT>(fmaf((x[2 * e] + sh[c]) * rs, g[c][2 * e], b[c][2 * e]),
                             fmaf((x[2 * e + 1] + sh[c]) * rs, g[c][2 * e + 1], b[c][2 * e + 1]));
      __stcg(reinterpret_cast<uint4*>(rowp + col), make_uint4(w[0], w[1], w[2], w[3]));
    }
  }
}

// Bandwidth-oriented row pass (large M, N <= 256 * kSlabs): one warp per row, the whole
// row loaded by one batch of 16-byte loads per lane (columns u * 256 + lane * 8), the
// statistics merged with shuffles only (no block barrier), gamma / beta read per slab
// at the end (they stay in L1 across the block's rows).  Same arithmetic as
// fo_ln_rows_kernel.
template <int OUT_DT, bool RESID, int kSlabs>
__global__ void __launch_bounds__(256) fo_ln_warp_rows_kernel(const KParams p, int bn) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * 8 + warp;
  griddep_wait();
  if (row >= p.M) return;
  unsigned short* rowp = reinterpret_cast<unsigned short*>(p.out) + row * p.ldo;
  uint4 y[kSlabs];
#pragma unroll
  for (int u = 0; u < kSlabs; ++u) {
    const int col = u * 256 + lane * 8;
    if (col < p.N) y[u] = __ldcg(reinterpret_cast<const uint4*>(rowp + col));
  }
  float mean, rs;
  float sh[kSlabs];
  if constexpr (RESID) {
    const unsigned short* resp = reinterpret_cast<const unsigned short*>(p.residual) + row * p.ldr;
    float sum = 0.f;
#pragma unroll
    for (int u = 0; u < kSlabs; ++u) {
      const int col = u * 256 + lane * 8;
      if (col < p.N) {
        const uint4 r = __ldg(reinterpret_cast<const uint4*>(resp + col));
        uint32_t wy[4] = {y[u].x, y[u].y, y[u].z, y[u].w};
        const uint32_t wr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {  // x = round16(y + residual), the reference's 16-bit add
          const float2 a = unpack2<OUT_DT>(wy[e]), b = unpack2<OUT_DT>(wr[e]);
          wy[e] = pack2<OUT_DT>(a.x + b.x, a.y + b.y);
          const float2 q = unpack2<OUT_DT>(wy[e]);
          sum += q.x + q.y;
        }
        y[u] = make_uint4(wy[0], wy[1], wy[2], wy[3]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    mean = sum / static_cast<float>(p.N);
    float q2 = 0.f;
#pragma unroll
    for (int u = 0; u < kSlabs; ++u) {
      if (u * 256 + lane * 8 < p.N) {
        const uint32_t wy[4] = {y[u].x, y[u].y, y[u].z, y[u].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 a = unpack2<OUT_DT>(wy[e]);
          q2 += (a.x - mean) * (a.x - mean) + (a.y - mean) * (a.y - mean);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q2 += __shfl_xor_sync(0xffffffffu, q2, o);
    rs = rsqrtf(q2 / static_cast<float>(p.N) + p.eps);
#pragma unroll
    for (int u = 0; u < kSlabs; ++u) sh[u] = -mean;
  } else {
    float shift[kSlabs];
#pragma unroll
    for (int u = 0; u < kSlabs; ++u) {
      const int col = u * 256 + lane * 8;
      shift[u] = col < p.N ? __ldcg(p.ln_stats + static_cast<long long>(col / bn) * p.M + row).z : 0.f;
    }
    float cnt = 0.f, m = 0.f, m2 = 0.f;
    for (int j = lane; j < p.tiles_n; j += 32) {
      const float4 pm = __ldcg(p.ln_stats + static_cast<long long>(j) * p.M + row);
      chan_merge(cnt, m, m2, static_cast<float>(min(bn, p.N - j * bn)), pm.x, pm.y);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float c2 = __shfl_xor_sync(0xffffffffu, cnt, o);
      const float mb = __shfl_xor_sync(0xffffffffu, m, o);
      const float m2b = __shfl_xor_sync(0xffffffffu, m2, o);
      chan_merge(cnt, m, m2, c2, mb, m2b);
    }
    mean = m;
    rs = rsqrtf(m2 / static_cast<float>(p.N) + p.eps);
#pragma unroll
    for (int u = 0; u < kSlabs; ++u) sh[u] = shift[u] - mean;
  }
#pragma unroll
  for (int u = 0; u < kSlabs; ++u) {
    const int col = u * 256 + lane * 8;
    if (col < p.N) {
      float g[8], b[8];
      load_vec8(p.gamma, p.vec_dtype, col, g);
      load_vec8(p.beta, p.vec_dtype, col, b);
      uint32_t w[4] = {y[u].x, y[u].y, y[u].z, y[u].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack2<OUT_DT>(w[e]);
        w[e] = pack2<OUT_DT>(fmaf((f.x + sh[u]) * rs, g[2 * e], b[2 * e]),
                             fmaf((f.y + sh[u]) * rs, g[2 * e + 1], b[2 * e + 1]));
      }
      __stcg(reinterpret_cast<uint4*>(rowp + col), make_uint4(w[0], w[1], w[2], w[3]));
    }
  }
}

}  // namespace fo

