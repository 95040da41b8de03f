// fo_direct.cuh -- direct convolution for stride-1 NHWC convs on sm_100a.
//
// The im2col kernel (fo_tc_kernel<..., CONV>) loads every input pixel once per filter
// tap from L2: a 3x3 conv moves 9x its input through each SM's load path, which bounds
// it well below the tensor rate.  Here each input pixel is loaded into shared memory
// once per 128-channel output tile and every tap is a shifted view of the same rows:
//
//   * The image is viewed with padded rows of P positions (P = W + 2*pad rounded up to
//     32).  Inside a tile, output position q = r * P + ow (r = output row of the tile)
//     and tap (dy, dx) reads padded-input position q + dy * P + dx, a constant shift.
//     Positions with ow >= OW or with an output row past OH are computed and discarded.
//   * A tile is rpt whole output rows of one image (BN = rpt * P <= 256 positions, rpt
//     chosen by the host so that the tiles cover OH with little waste and fill the
//     waves evenly) x 128 output channels (operand-swapped: M = channels from the
//     weights, N = positions).  The slot producer loads the nR padded rows the tile's
//     taps touch, one 4-D TMA box of (64 channels, P positions) per row starting at
//     w = -pad (the padding, and rows past the image, are the hardware's out-of-range
//     zero fill; every box lands 1024-byte aligned because P * 128 B is a multiple of
//     4 KB).
//   * For each channel block and tap the MMA issuer points the B descriptor at the rows
//     shifted by dy * P + dx positions (128 B each); the swizzle is anchored on absolute
//     shared-memory addresses, so any row shift is a plain start-address offset.
//   * The weights stream through a ring of 128 x 64 stages (one or two taps per stage)
//     from their own producer thread; the pixel slots have a producer thread of their
//     own (the last warp), so a slot is refilled as soon as it frees instead of after the
//     weight loads queued before it.
//   * Eight epilogue warps (two per TMEM lane quarter) take 32-position chunks: with
//     P % 32 == 0 each chunk is part of one padded row, stored with one 4-D TMA box
//     (32 channels x 32 columns) whose out-of-range columns the hardware clips.
// Per 128 x BN x 64 MMA step an SM loads 16 KB of weights plus 1/(KH*KW) of the rows
// instead of 16 KB + BN * 128 B.  Every wait is bounded as in fo_tc_kernel.
#pragma once
#include "fo_kernel.cuh"

namespace fo {

constexpr int kDirectMaxBN = 256;       // positions per tile, at most
constexpr int kDirectThreads = 352;     // weight producer, MMA, 8 epilogue, slot producer
constexpr int kDirectWStage = 128 * 64 * 2;  // 128 channels x 64 K of weights

// kps: filter taps per weight stage (1; 2 = block_k 128; 3 = block_k 192).  More MMAs
// per barrier wait (8 or 12 instead of 4) cost fewer waits but allow fewer, larger
// stages; with the warp-uniform issue loop below one tap per stage and six stages
// measure as fast as two taps x three stages on 28 x 28 images.
__host__ __device__ constexpr int direct_smem_bytes(int stages, int pslots, int slot_bytes, int kps = 1) {
  return 1024 + pslots * slot_bytes + stages * kps * kDirectWStage + kEpiBytes + kMiscBytes;
}

template <int ACT, int OUT_DT, int KPS = 1>
__global__ void __launch_bounds__(kDirectThreads, 1)
    fo_direct_conv_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                          const __grid_constant__ CUtensorMap tmY, const KParams p) {
  constexpr int kMmaWarp = 1, kFirstEpiWarp = 2, kSlotWarp = kFirstEpiWarp + kEpiWarps;
  const int BN = p.rpt * p.P;  // positions per tile
  constexpr int kOutBytes = OUT_DT == DT_F32 ? 4 : 2;
  constexpr uint32_t kTmemCols = 2 * kDirectMaxBN;  // two accumulators, 256 columns apart

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int stages = p.stages;
  const int slot_bytes = p.nR * p.P * 128;
  const uint32_t sPix = smem_u32(smem);
  const uint32_t sW = sPix + p.pslots * slot_bytes;
  const uint32_t sEpi = sW + stages * KPS * kDirectWStage;
  uint8_t* misc = smem + (sEpi - sPix) + kEpiBytes;
  // misc: [0,64) full[8] | [64,128) empty[8] | [128,144) pfull[2] | [144,160) pempty[2]
  //       | [160,176) tfull[2] | [176,192) tempty[2] | [192,200) drain | [248,256) tmem addr + abort
  const uint32_t mb = smem_u32(misc);
  const uint32_t bar_full = mb, bar_empty = mb + 64, bar_pfull = mb + 128, bar_pempty = mb + 144;
  const uint32_t bar_tfull = mb + 160, bar_tempty = mb + 176, bar_drain = mb + 192;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 248);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 252);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cid = blockIdx.x, ncl = gridDim.x;
  const uint64_t tmo = p.timeout_ns;
  const int taps = p.KH * p.KW;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_pfull + 8 * a, 1);
      mbar_init(bar_pempty + 8 * a, 1);
      mbar_init(bar_tfull + 8 * a, 1);
      mbar_init(bar_tempty + 8 * a, kEpiWarps);
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  if (threadIdx.x == 32 * kFirstEpiWarp) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmY);
  }
  __syncwarp();  // reconverge each warp before the CTA-wide barrier
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ weight producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int issued = 0;
      bool ok = true;
      for (int u = cid; u < p.num_units && ok; u += ncl) {
        const int tm = u % p.tiles_m;
        for (int cb = 0; cb < p.c_blocks && ok; ++cb) {
          for (int t = 0; t < taps; t += KPS) {
            const int nk = KPS == 1 ? 1 : min(KPS, taps - t);  // taps in this stage
            if (!mbar_wait(bar_empty + 8 * s, ph ^ 1, tmo, abort_flag)) {
              ok = false;
              break;
            }
            const uint32_t fb = bar_full + 8 * s;
            mbar_arrive_expect_tx(fb, nk * kDirectWStage);
            for (int i = 0; i < nk; ++i) {
#pragma unroll
              for (int j = 0; j < 2; ++j)  // 128 output channels x 64 K, MN-major
                tma_load_2d(sW + (s * KPS + i) * kDirectWStage + j * 64 * 128, &tmW, fb, tm * 128 + j * 64,
                            (t + i) * p.C + cb * 64);
            }
            ++issued;
            if (++s == stages) {
              s = 0;
              ph ^= 1;
            }
          }
        }
      }
      if (!ok) {
        record_error(p, kStatusTimeout, 0x40);
        *abort_flag = 1;
      }
      drain_loads(bar_full, stages, issued);
    }
  } else if (warp == kSlotWarp) {
    // ------------------------------------------------------------------ slot producer
    if (lane == 0) {
      int ps = 0;
      uint32_t pph = 0;
      int pissued = 0;
      bool ok = true;
      const uint32_t row_bytes = static_cast<uint32_t>(p.P) * 128;
      for (int u = cid; u < p.num_units && ok; u += ncl) {
        const int tn = u / p.tiles_m;
        const int n = tn / p.tpi;
        const int hp0 = (tn - n * p.tpi) * p.rpt;  // first padded input row = first output row
        for (int cb = 0; cb < p.c_blocks; ++cb) {
          if (!mbar_wait(bar_pempty + 8 * ps, pph ^ 1, tmo, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t pb = bar_pfull + 8 * ps;
          mbar_arrive_expect_tx(pb, static_cast<uint32_t>(p.nR) * row_bytes);
          for (int r = 0; r < p.nR; ++r)  // rows past the image are zero-filled
            tma_load_4d(sPix + ps * slot_bytes + r * row_bytes, &tmX, pb, cb * 64, -p.pad, hp0 + r - p.pad, n);
          ++pissued;
          if (++ps == p.pslots) {
            ps = 0;
            pph ^= 1;
          }
        }
      }
      if (!ok) {
        record_error(p, kStatusTimeout, 0x43);
        *abort_flag = 1;
      }
      drain_loads(bar_pfull, p.pslots, pissued);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs this loop and lane 0 alone waits, issues and commits (elect.sync
    // inside the MMA / commit instructions), so the loop's control flow and descriptor
    // arithmetic stay warp-uniform.  The issuing lane is the bottleneck of this loop (each
    // tcgen05.mma takes ~60 issue cycles, a commit ~60, against 448 tensor cycles per tap),
    // so every descriptor is stepped, not recomputed: the weights by one stage (16 KB) per
    // tap, the rows by one position (128 B) per dx and by P - KW + 1 positions at the end
    // of a filter row.
    auto wait = [&](uint32_t bar, uint32_t parity) {
      int r = 1;
      if (lane == 0) r = mbar_wait(bar, parity, tmo, abort_flag) ? 1 : 0;
      return __shfl_sync(0xffffffffu, r, 0) != 0;
    };
    const uint32_t idesc = idesc_f16(p.ab_bf16, 0, BN, 128) | (1u << 15);  // A (weights) MN-major
    const uint64_t a_desc0 = sdesc_sw128(sW, 64 * 128, 1024);
    const uint64_t b_desc0 = sdesc_sw128_rows(sPix);
    const uint32_t slot_units = static_cast<uint32_t>(slot_bytes) >> 4;
    const uint32_t wrap_units = static_cast<uint32_t>(p.P - p.KW + 1) * 8;
    int s = 0, ps = 0, acc = 0;
    uint32_t ph = 0, pph = 0, acc_ph = 0;
    uint64_t ad = a_desc0;
    bool ok = true;
    for (int u = cid; u < p.num_units && ok; u += ncl) {
      if (!wait(bar_tempty + 8 * acc, acc_ph ^ 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem_base + acc * kDirectMaxBN;
      uint32_t accum = 0;
      for (int cb = 0; cb < p.c_blocks && ok; ++cb) {
        if (!wait(bar_pfull + 8 * ps, pph)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint64_t bd = b_desc0 + static_cast<uint64_t>(ps * slot_units);
        int dx = 0;
        for (int t = 0; t < taps; t += KPS) {
          const int nk = KPS == 1 ? 1 : min(KPS, taps - t);
          if (!wait(bar_full + 8 * s, ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int i = 0; i < KPS; ++i) {
            if (KPS > 1 && i >= nk) break;
            const uint64_t a = ad + static_cast<uint64_t>(i * (kDirectWStage >> 4));
            tc_mma_f16_x4_elect(d, a, bd, idesc, accum, 2048 >> 4, 32 >> 4);
            accum = 1u;
            if (++dx == p.KW) {
              dx = 0;
              bd += wrap_units;
            } else {
              bd += 8;
            }
          }
          tc_commit_elect(bar_empty + 8 * s);
          if (++s == stages) {
            s = 0;
            ph ^= 1;
            ad = a_desc0;
          } else {
            ad += KPS * (kDirectWStage >> 4);
          }
        }
        tc_commit_elect(bar_pempty + 8 * ps);
        if (++ps == p.pslots) {
          ps = 0;
          pph ^= 1;
        }
      }
      if (!ok) break;
      tc_commit_elect(bar_tfull + 8 * acc);
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1;
    }
    if (lane == 0) {
      if (!ok) {
        record_error(p, kStatusTimeout, 0x41);
        *abort_flag = 1;
      }
      tc_commit(bar_drain);
      mbar_wait(bar_drain, 0, kDrainTimeoutNs, nullptr);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int ew = warp - kFirstEpiWarp;  // 0..7
    const int quarter = warp & 3;         // TMEM lane quarter = 32 output channels
    const int half = ew >> 2;             // 128-position half of the tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t buf0 = sEpi + ew * kEpiBufBytes;
    constexpr int kRowB = 32 * kOutBytes;  // one staged pixel: 32 channels
    constexpr int kBox = 32 * kRowB;
    constexpr int kBufs = kEpiBufBytes / kBox;
    int acc = 0;
    uint32_t acc_ph = 0, nstore = 0;
    bool ok = true;
    for (int u = cid; u < p.num_units; u += ncl) {
      const int tm = u % p.tiles_m, tn = u / p.tiles_m;
      const int f0 = tm * 128 + quarter * 32;
      const int f = f0 + lane;
      const float2 aff = channel_affine(p, f);
      const bool has_add = OUT_DT != DT_F32 && p.add_src != nullptr && f0 < p.N;
      const int n = tn / p.tpi;
      const int oh0 = (tn - n * p.tpi) * p.rpt;
      // the tile's BN / 32 chunks: the first half of the warps takes chunks 0-3, the second
      // half the rest (none when BN <= 128: those warps only release the accumulator)
      const int mine = min(4, max(0, BN / 32 - half * 4));
      // Residual of chunk c (32 positions of one padded row): lane = pixel ow0 + lane, its
      // 32 channels as 4 x 16 B; zeros for padding positions and absent channels.  It does
      // not depend on the accumulator, so the first chunk's is loaded before the wait and
      // each next chunk's while the current one is processed.
      auto load_res = [&](int c, uint4 (&q)[4]) {
#pragma unroll
        for (int j = 0; j < 4; ++j) q[j] = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (OUT_DT != DT_F32) {
          const int pos0 = c * 32;
          const int rr = pos0 / p.P;
          const int oh = oh0 + rr;
          const int ow = pos0 - rr * p.P + lane;
          if (!has_add || oh >= p.OH || ow >= p.OW) return;
          const unsigned short* src = reinterpret_cast<const unsigned short*>(p.add_src) +
                                      ((static_cast<long long>(n) * p.OH + oh) * p.OW + ow) * p.ld_add + f0;
          if (f0 + 32 <= p.N) {
#pragma unroll
            for (int j = 0; j < 4; ++j) q[j] = __ldg(reinterpret_cast<const uint4*>(src) + j);
          } else {  // partial channel group
            unsigned short tmp[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) tmp[e] = f0 + e < p.N ? src[e] : static_cast<unsigned short>(0);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              q[j] = make_uint4(tmp[8 * j] | (tmp[8 * j + 1] << 16), tmp[8 * j + 2] | (tmp[8 * j + 3] << 16),
                                tmp[8 * j + 4] | (tmp[8 * j + 5] << 16), tmp[8 * j + 6] | (tmp[8 * j + 7] << 16));
          }
        }
      };
      uint4 qn[4] = {};
      if (has_add && mine > 0) load_res(half * 4, qn);
      if (!mbar_wait(bar_tfull + 8 * acc, acc_ph, tmo, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (mine == 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_tempty + 8 * acc);
      }
#pragma unroll 1
      for (int ci = 0; ci < mine; ++ci) {
        const int c = half * 4 + ci;
        uint4 q[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) q[j] = qn[j];
        if (has_add && ci + 1 < mine) load_res(c + 1, qn);
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + lane_off + acc * kDirectMaxBN + c * 32, r);
        tc_wait_ld_regs(r);
        if (ci == mine - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_tempty + 8 * acc);
        }
        const int pos0 = c * 32;  // 32 positions inside one padded row of the tile
        const int rr = pos0 / p.P;
        const int oh = oh0 + rr;
        const int ow0 = pos0 - rr * p.P;
        if (oh >= p.OH || ow0 >= p.OW || f0 >= p.N) continue;  // padding positions
        float acc_v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc_v[i] = __uint_as_float(r[i]);
        if (p.bn_mode) {
#pragma unroll
          for (int i = 0; i < 32; ++i) acc_v[i] = fmaf(round_in(acc_v[i], p.ab_bf16), aff.x, aff.y);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) acc_v[i] = fmaf(acc_v[i], aff.x, aff.y);
        }
        const uint32_t buf = buf0 + (nstore % kBufs) * kBox;
        if (nstore >= kBufs) {
          if (lane == 0) bulk_wait_read<kBufs - 1>();
          __syncwarp();
        }
        if constexpr (OUT_DT != DT_F32) {
          if (has_add) {
            // residual (loaded ahead, q): transposed through the staging block it will be
            // stored from
#pragma unroll
            for (int j = 0; j < 4; ++j)
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(buf + lane * kRowB + j * 16), "r"(q[j].x),
                           "r"(q[j].y), "r"(q[j].z), "r"(q[j].w)
                           : "memory");
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              unsigned short h;
              asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(buf + i * kRowB + lane * 2) : "memory");
              acc_v[i] += unpack2<OUT_DT>(static_cast<uint32_t>(h)).x;
            }
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
          tma_store_4d(&tmY, buf, f0, ow0, oh, n);
          bulk_commit();
        }
        ++nstore;
      }
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1;
    }
    if (!ok) {
      record_error(p, kStatusTimeout, 0x42);
      *abort_flag = 1;
    }
    if (lane == 0) bulk_wait_read<0>();  // the stores complete with the grid
    __syncwarp();
  }

  __syncwarp();  // the producer and MMA warps ran their loops on lane 0 alone
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace fo
