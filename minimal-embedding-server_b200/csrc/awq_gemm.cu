// AWQ W4A16 GEMM on tcgen05 / TMEM, plus the load-time repack and a standalone
// dequantiser that shares the GEMM's arithmetic.
//
// Y[M, N] = X[M, K] * W[K, N] (+ bias), W[k, n] = bf16_rne((q - z) * s).
//
// The product is computed transposed, Y^T = W^T X^T, so that the dequantised weights are
// the MMA's A operand (128 features per CTA) and the tokens its N dimension.  Every kernel
// here has the same roles:
//   * a TMA warp streams X tiles (BT tokens x 64 k, bf16, 128-byte swizzle), the packed
//     weight tile (8 words x 128 features of the kernel layout) and the group's scales and
//     zero words into a ring of shared-memory stages;
//   * dequant warps (one output feature per thread) turn 8 words = 64 k of their feature
//     into 32 bf16x2 values and store them as the step's A tile - into TMEM with tcgen05.st
//     (small-M kernel) or into shared memory with the 128-byte swizzle (persistent and
//     CTA-pair kernels); the bf16 weights never reach HBM;
//   * one thread issues tcgen05.mma (M = 128 features, or 256 across a CTA pair; N = BT
//     tokens; K = 16), accumulating fp32 in TMEM, and frees each stage with tcgen05.commit;
//   * epilogue warps drain the accumulator (tcgen05.ld) and add the bias, then write bf16
//     through shared memory with TMA stores, add into an fp32 residual, or apply
//     SiLU-and-mul.
// Which kernel runs for which M, N and epilogue is decided in dispatch_gemm.
//
// Exact dequantisation in bf16x2 arithmetic: the code pair (q_k, q_k+1) is extracted as the
// bf16 pair (128 + q) with one LOP3 (the nibble interleave puts k and k+1 at bits 4j and
// 16 + 4j); subtracting (128 + z) is exact; the fp16 scale is split into s_hi = bf16(s) and
// s_lo = bf16(s - s_hi) (exact, <= 3 significant bits), (q - z) * s_lo is exact in bf16,
// and fma.rn(q - z, s_hi, (q - z) * s_lo) rounds (q - z) * s exactly once.
#include "common.cuh"

namespace {

__device__ int g_err_gemm = 0;

// Epilogue modes of the GEMM kernels.
//   kEpiBf16:     Y = bf16(acc + bias)
//   kEpiResidual: R (fp32) += acc + bias      (o_proj / down_proj into the residual stream)
//   kEpiSilu:     Y = bf16(silu(gate) * up)   (gate_up with SiLU-and-mul; the weight columns
//                 are interleaved in blocks of 16 - columns [32b, 32b+16) hold gate features
//                 16b.., [32b+16, 32b+32) the matching up features - so every TMEM lane
//                 quadrant holds both halves of its 16 outputs; Y has N/2 columns)
constexpr int kEpiBf16 = 0, kEpiResidual = 1, kEpiSilu = 2;


// SiLU-and-mul epilogue of one chunk of CHUNK tokens for one warp.  Lane l < 16 holds the
// gate feature and lane l + 16 the matching up feature of output column `x + l`; one
// shuffle per token pair gives lane l the up values of the first half of the chunk and
// lane l + 16 the gate values of the second half, so each lane produces CHUNK / 2 outputs.
template <int CHUNK>
__device__ __forceinline__ void silu_chunk(const uint32_t (&v)[CHUNK], int lane,
                                           __nv_bfloat16* buf, bool& stored,
                                           const CUtensorMap* map_y, int x, int y) {
  constexpr int H = CHUNK / 2;
  const bool lo = lane < 16;
  const int f = lane & 15;
  if (stored) {
    if (lane == 0) mes::tma_store_wait_read<0>();
    __syncwarp();
  }
#pragma unroll
  for (int j = 0; j < H; ++j) {
    // lo lanes send their gate value of token H + j and receive the up value of token j.
    const float send = __uint_as_float(lo ? v[H + j] : v[j]);
    const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
    const float g = lo ? __uint_as_float(v[j]) : recv;
    const float u = lo ? recv : __uint_as_float(v[H + j]);
    // silu(g) = g / (1 + e^-g); the approximate divide needs no special-case path, and for
    // g < -88 (e^-g = inf) it returns 0, the limit of silu.
    const float o = __fdividef(g, 1.0f + __expf(-g)) * u;
    buf[((lo ? 0 : H) + j) * 16 + f] = __float2bfloat16_rn(o);
  }
  mes::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    mes::tma_store_2d(map_y, buf, x, y);
    mes::tma_store_commit();
  }
  __syncwarp();
  stored = true;
}

constexpr int kBN = 128;  // output features per tile (MMA M)
constexpr int kBK = 64;   // k per pipeline stage (one 128-byte swizzle row of bf16)
constexpr int kGroup = 128;

// Position of column (n % 8) inside an AWQ-packed word.
__constant__ int kInvOrder[8] = {0, 4, 1, 5, 2, 6, 3, 7};

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

struct GroupParams {
  uint32_t zz2;   // bf16x2 {128 + z, 128 + z}
  uint32_t shi2;  // bf16x2 {s_hi, s_hi}
  uint32_t slo2;  // bf16x2 {s_lo, s_lo}
};

__device__ __forceinline__ GroupParams make_group(uint32_t zword, int zshift, uint16_t sbits) {
  GroupParams g;
  const uint32_t z = (zword >> zshift) & 0xFu;
  g.zz2 = (0x4300u | z) * 0x00010001u;
  const float s = __half2float(__ushort_as_half(sbits));
  const __nv_bfloat16 hi = __float2bfloat16_rn(s);
  const __nv_bfloat16 lo = __float2bfloat16_rn(s - __bfloat162float(hi));
  g.shi2 = (uint32_t)__bfloat16_as_ushort(hi) * 0x00010001u;
  g.slo2 = (uint32_t)__bfloat16_as_ushort(lo) * 0x00010001u;
  return g;
}

// bf16 pair (k, k+1) from a kernel-layout word already shifted right by 4j.
__device__ __forceinline__ uint32_t dq_pair(uint32_t w, const GroupParams& g) {
  const uint32_t v = (w & 0x000F000Fu) | 0x43004300u;
  const uint32_t d = bf16x2_sub(v, g.zz2);
  return bf16x2_fma(d, g.shi2, bf16x2_mul(d, g.slo2));
}

// ----------------------------------------------------------------------------------------
// One tile per CTA (small M): BT tokens (the MMA's N), STAGES shared-memory stages, ASLOTS
// dequantised-A slots in TMEM, NDQ dequant/epilogue warps (4: one per TMEM lane quadrant;
// 8: two per quadrant, each taking half of a stage's words and half of the epilogue's token
// chunks).  Each stage holds the X tile, the packed weight words and the group's scales and
// zero words (all by TMA).  Small tiles stream little data per k-step, so the ring is deep
// (about 100 KB in flight per CTA) to cover the HBM latency, while TMEM keeps only a few A
// slots.
//
// Split-K over a cluster.  With split > 1 the grid is launched in clusters of `split` CTAs
// along x, all on the same 128-feature x BT-token tile; CTA r runs the weight groups
// [r G / split, (r + 1) G / split) of the G = K / 128 groups.  After the mainloop each CTA
// writes its fp32 partial tile into its stage ring (idle by then), the cluster
// synchronises, and the tile's (lane quadrant, token chunk) units are dealt out over the
// cluster: the CTA owning a unit reads that unit of all `split` partial tiles through
// distributed shared memory, adds them in rank order (so the sum does not depend on which
// CTA reduces) and runs the epilogue.  A second cluster barrier keeps every CTA's shared
// memory alive until all reads are done.  No global workspace and no atomics: the result
// is deterministic.
template <int BT, int STAGES, int ASLOTS, int EPI, int NDQ>
struct Cfg {
  static constexpr bool kResidual = EPI == kEpiResidual, kSilu = EPI == kEpiSilu;
  static constexpr int kThreads = 64 + 32 * NDQ;  // warp 0 TMA, warp 1 MMA, then NDQ warps
  static constexpr int kHalves = NDQ / 4;
  static constexpr int kWords = 8 / kHalves;      // packed words per dequant thread per stage
  static constexpr int kXStage = BT * kBK * 2;
  static constexpr int kWBytes = (kBK / 8) * kBN * 4;  // 8 words x 128 features
  static constexpr int kWStage = kWBytes + 256 + 128;  // words | scales (256 B) | zeros (64 B)
  static constexpr int kChunk = kResidual ? 16 : (BT < 32 ? BT : 32);  // tokens per epilogue step
  static constexpr int kOutBuf = kChunk * 32 * 2;  // one staging block per epilogue warp
  static constexpr int kOffX = 0;
  static constexpr int kOffW = STAGES * kXStage;
  static constexpr int kOffOut = kOffW + STAGES * kWStage;
  static constexpr int kOffBar = kOffOut + (kResidual ? 0 : NDQ * kOutBuf);
  static constexpr int kSmem = kOffBar + 512 + 1024;  // barriers + 1 KB alignment slack
  static constexpr int kRedBytes = BT * kBN * 4;      // one fp32 partial tile (split-K)
  static constexpr int kTmemNeed = BT + ASLOTS * 32;
  static constexpr int kTmemCols = kTmemNeed <= 32 ? 32 : kTmemNeed <= 64 ? 64
                                 : kTmemNeed <= 128 ? 128 : kTmemNeed <= 256 ? 256 : 512;
  // Shared memory requested at launch: at least enough that no more CTAs fit on an SM
  // (228 KB, 1 KB reserved per CTA) than its 512 TMEM columns serve at once, so that no CTA
  // waits in tcgen05.alloc for another; with split-K such a wait could close a cycle
  // through the cluster barriers.  The launcher checks the resulting occupancy.
  static constexpr int kCtasByTmem = 512 / kTmemCols;
  static constexpr int kSmemFloor = 233472 / (kCtasByTmem + 1) - 1024 + 1;
  static constexpr int kSmemLaunch = kSmem > kSmemFloor ? kSmem : kSmemFloor;
  static_assert(NDQ == 4 || NDQ == 8, "dequant warps");
  static_assert(kTmemNeed <= 512, "TMEM budget");
  static_assert(kSmemLaunch <= 232448, "shared memory budget");
  static_assert(BT % 16 == 0 && BT >= 16 && BT <= 256, "MMA N");
  static_assert(kXStage % 1024 == 0 && kWStage % 128 == 0, "stage alignment");
  static_assert(kRedBytes <= kOffOut, "the partial tile fits in the stage ring");
  static_assert((2 * STAGES + 2 * ASLOTS + 1) * 8 + 8 <= 512, "barrier area");
  static_assert(kChunk % 4 == 0, "partial tiles are stored four tokens per 16 bytes");
};

// EPI selects the epilogue (kEpiBf16 / kEpiResidual / kEpiSilu, see their definition).
template <int BT, int STAGES, int ASLOTS, int EPI, int NDQ>
__global__ void __launch_bounds__(Cfg<BT, STAGES, ASLOTS, EPI, NDQ>::kThreads)
awq_gemm_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                const __grid_constant__ CUtensorMap map_s, const __grid_constant__ CUtensorMap map_z,
                const __grid_constant__ CUtensorMap map_y, const __nv_bfloat16* __restrict__ bias,
                float* __restrict__ R, int64_t ldr, int M, int N, int K, int split) {
  using C = Cfg<BT, STAGES, ASLOTS, EPI, NDQ>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem + C::kOffX;
  uint8_t* wst = smem + C::kOffW;
  float* red = reinterpret_cast<float*>(smem);  // partial tile over the ring (split > 1)
  __nv_bfloat16* outbuf = reinterpret_cast<__nv_bfloat16*>(smem + C::kOffOut);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* full = bars;                  // [STAGES] TMA landed (X, words, scales, zeros)
  uint64_t* empty = bars + STAGES;        // [STAGES] MMAs of the stage done
  uint64_t* afull = bars + 2 * STAGES;    // [ASLOTS] dequantised A written to TMEM
  uint64_t* aempty = afull + ASLOTS;      // [ASLOTS] MMAs reading the A slot done
  uint64_t* accum = aempty + ASLOTS;      // all MMAs done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = mes::warp_id(), lane = mes::lane_id();
  const int rank = split > 1 ? static_cast<int>(mes::cluster_ctarank()) : 0;
  const int n0 = (blockIdx.x / split) * kBN;
  const int t0 = blockIdx.y * BT;
  // This CTA's k-steps: whole groups (two 64-k steps each), split as evenly as they go.
  const int groups = K / kGroup;
  const int kb0 = 2 * (rank * groups / split);
  const int nloc = 2 * ((rank + 1) * groups / split) - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mes::mbar_init(&full[s], 1);
      mes::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < ASLOTS; ++a) {
      mes::mbar_init(&afull[a], NDQ);
      mes::mbar_init(&aempty[a], 1);
    }
    mes::mbar_init(accum, 1);
    *abort_flag = 0;
    mes::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    mes::tma_prefetch_desc(&map_x);
    mes::tma_prefetch_desc(&map_w);
    mes::tma_prefetch_desc(&map_s);
    mes::tma_prefetch_desc(&map_z);
    if (!C::kResidual) mes::tma_prefetch_desc(&map_y);
  }
  if (warp == 1) {
    __syncwarp();
    mes::tmem_alloc(tmem_slot, C::kTmemCols);
    mes::tmem_relinquish();
  }
  mes::tc_fence_before();
  __syncthreads();
  mes::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_a = tmem + BT;  // A slots after the BT accumulator columns

  // Epilogue of one chunk of C::kChunk tokens at token offset c0 of the tile, for the 32
  // features of lane quadrant q (v[j] = fp32 bits of token c0 + j, feature of this lane).
  const int q = warp & 3;
  const int row = q * 32 + lane;  // feature within the tile (dequant / epilogue warps)
  const int n = n0 + row;
  const float bv = (warp >= 2 && bias) ? __bfloat162float(bias[n]) : 0.f;
  __nv_bfloat16* buf = outbuf + (warp >= 2 ? warp - 2 : 0) * (C::kOutBuf / 2);
  bool stored = false;
  auto store_chunk = [&](const uint32_t (&v)[C::kChunk], int c0) {
    if constexpr (C::kSilu) {
      silu_chunk<C::kChunk>(v, lane, buf, stored, &map_y, n0 / 2 + q * 16, t0 + c0);
    } else if constexpr (C::kResidual) {
      // Each lane owns feature n; a warp touches 32 consecutive fp32 per token row.
      const int rows = min(C::kChunk, M - (t0 + c0));
      float* rp = R + (int64_t)(t0 + c0) * ldr + n;
      float rv[C::kChunk];
#pragma unroll
      for (int j = 0; j < C::kChunk; ++j) rv[j] = j < rows ? rp[(int64_t)j * ldr] : 0.f;
#pragma unroll
      for (int j = 0; j < C::kChunk; ++j)
        if (j < rows) rp[(int64_t)j * ldr] = rv[j] + (__uint_as_float(v[j]) + bv);
    } else {
      if (stored) {  // the previous TMA store must have read the staging block
        if (lane == 0) mes::tma_store_wait_read<0>();
        __syncwarp();
      }
#pragma unroll
      for (int j = 0; j < C::kChunk; ++j)
        buf[j * 32 + lane] = __float2bfloat16_rn(__uint_as_float(v[j]) + bv);
      mes::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mes::tma_store_2d(&map_y, buf, n0 + q * 32, t0 + c0);
        mes::tma_store_commit();
      }
      __syncwarp();
      stored = true;
    }
  };
  auto load_acc = [&](uint32_t (&v)[C::kChunk], int c0) {
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    if constexpr (C::kChunk == 32) mes::tmem_ld32(tmem + lane_off + c0, v);
    else mes::tmem_ld16(tmem + lane_off + c0, v);
    mes::tmem_wait_ld();
  };

  bool epi_ok = false;  // this warp's accumulator is complete (dequant / epilogue warps)
  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nloc; ++i) {
        const int s = i % STAGES, kb = kb0 + i;
        if (i >= STAGES &&
            !mes::mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT))
          break;
        uint8_t* w = wst + s * C::kWStage;
        mes::mbar_arrive_expect_tx(&full[s], C::kXStage + C::kWBytes + 256 + 64);
        mes::tma_load_2d(xs + s * C::kXStage, &map_x, &full[s], kb * kBK, t0);
        mes::tma_load_2d(w, &map_w, &full[s], n0, kb * (kBK / 8));
        mes::tma_load_2d(w + C::kWBytes, &map_s, &full[s], n0, kb / 2);
        mes::tma_load_2d(w + C::kWBytes + 256, &map_z, &full[s], n0 / 8, kb / 2);
        issued = i + 1;
      }
      if (*abort_flag) {
        // Let the copies already issued land before the CTA exits.
        for (int i = issued - STAGES < 0 ? 0 : issued - STAGES; i < issued; ++i) {
          const uint64_t tstart = mes::globaltimer_ns();
          while (!mes::mbar_try_wait(&full[i % STAGES], (i / STAGES) & 1) &&
                 mes::globaltimer_ns() - tstart < mes::kWaitLimitNs) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------- MMA issuer ---------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = mes::idesc_bf16_f32(kBN, BT, false);
      const uint32_t xs_addr = mes::smem_u32(xs);
      for (int i = 0; i < nloc; ++i) {
        const int s = i % STAGES, a = i % ASLOTS;
        // afull implies full: every dequant warp waited for the whole stage (X included)
        // before arriving.
        if (!mes::mbar_wait(&afull[a], (i / ASLOTS) & 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT)) break;
        mes::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t bdesc =
              mes::smem_desc_sw128(xs_addr + s * C::kXStage + kk * 32, 16, 1024);
          mes::mma_ts(tmem, tmem_a + a * 32 + kk * 8, bdesc, idesc, (i | kk) != 0);
        }
        mes::tc_commit(&empty[s]);
        mes::tc_commit(&aempty[a]);
      }
      mes::tc_commit(accum);
      if (*abort_flag) {
        const uint64_t tstart = mes::globaltimer_ns();
        while (!mes::mbar_try_wait(accum, 0) && mes::globaltimer_ns() - tstart < mes::kWaitLimitNs) {
        }
      }
    }
    __syncwarp();
  } else if (warp < 2 + NDQ) {
    // --------------------------- dequant + epilogue warps -----------------------------
    const int half = (warp - 2) / 4;        // which half of the words / token chunks
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int zshift = 4 * kInvOrder[row & 7];  // n0 is a multiple of 128
    bool ok = true;
    for (int i = 0; i < nloc; ++i) {
      const int s = i % STAGES, a = i % ASLOTS;
      if (!mes::mbar_wait_warp(&full[s], (i / STAGES) & 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT) ||
          (i >= ASLOTS &&
           !mes::mbar_wait_warp(&aempty[a], ((i / ASLOTS) & 1) ^ 1, abort_flag, &g_err_gemm,
                                MES_ERR_TIMEOUT))) {
        ok = false;
        break;
      }
      mes::tc_fence_after();
      const uint8_t* w = wst + s * C::kWStage;
      const GroupParams gp =
          make_group(reinterpret_cast<const uint32_t*>(w + C::kWBytes + 256)[row >> 3], zshift,
                     reinterpret_cast<const uint16_t*>(w + C::kWBytes)[row]);
      const uint32_t* wsrc = reinterpret_cast<const uint32_t*>(w) + half * C::kWords * kBN + row;
      uint32_t av[4 * C::kWords];
#pragma unroll
      for (int j = 0; j < C::kWords; ++j) {
        const uint32_t wv = wsrc[j * kBN];
        av[4 * j + 0] = dq_pair(wv, gp);
        av[4 * j + 1] = dq_pair(wv >> 4, gp);
        av[4 * j + 2] = dq_pair(wv >> 8, gp);
        av[4 * j + 3] = dq_pair(wv >> 12, gp);
      }
      if constexpr (C::kWords == 8) mes::tmem_st32(tmem_a + a * 32 + lane_off, av);
      else mes::tmem_st16(tmem_a + a * 32 + half * 16 + lane_off, av);
      mes::tmem_wait_st();
      mes::tc_fence_before();
      __syncwarp();
      if (lane == 0) mes::mbar_arrive(&afull[a]);
      __syncwarp();
    }
    epi_ok = ok && mes::mbar_wait_warp(accum, 0, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT);
    if (epi_ok) mes::tc_fence_after();
    if (epi_ok && split == 1) {
#pragma unroll 1
      for (int c0 = half * C::kChunk; c0 < BT; c0 += C::kHalves * C::kChunk) {
        if (t0 + c0 >= M) break;  // rows past the end of X: nothing to store
        uint32_t v[C::kChunk];
        load_acc(v, c0);
        store_chunk(v, c0);
      }
    }
  }

  if (split > 1) {
    // ------------------------------ split-K reduction ---------------------------------
    // Partial tile layout: token j, feature f at float index ((j / 4) * 128 + f) * 4 + j % 4,
    // so one lane's four consecutive tokens are one 16-byte word and a warp's 32 features
    // are 512 contiguous bytes.
    const int half = warp >= 2 ? (warp - 2) / 4 : 0;
    if (warp >= 2 && epi_ok) {
      mes::fence_proxy_async_smem();  // the ring was last written by TMA
#pragma unroll 1
      for (int c0 = half * C::kChunk; c0 < BT; c0 += C::kHalves * C::kChunk) {
        if (t0 + c0 >= M) break;
        uint32_t v[C::kChunk];
        load_acc(v, c0);
#pragma unroll
        for (int j = 0; j < C::kChunk; j += 4)
          *reinterpret_cast<float4*>(red + (((c0 + j) / 4) * kBN + row) * 4) =
              make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                          __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
      }
    }
    mes::cluster_sync();
    if (warp >= 2 && epi_ok) {
      const uint32_t red_addr = mes::smem_u32(red);
#pragma unroll 1
      for (int c0 = half * C::kChunk; c0 < BT; c0 += C::kHalves * C::kChunk) {
        if (t0 + c0 >= M) break;
        if (((c0 / C::kChunk) * 4 + q) % split != rank) continue;
        float acc[C::kChunk];
#pragma unroll 1
        for (int p = 0; p < split; ++p) {
          const uint32_t base = mes::mapa_shared(red_addr, (uint32_t)p);
#pragma unroll
          for (int j = 0; j < C::kChunk; j += 4) {
            const float4 f = mes::ld_dsmem_f4(base + (uint32_t)((((c0 + j) / 4) * kBN + row) * 16));
            if (p == 0) {
              acc[j] = f.x; acc[j + 1] = f.y; acc[j + 2] = f.z; acc[j + 3] = f.w;
            } else {
              acc[j] += f.x; acc[j + 1] += f.y; acc[j + 2] += f.z; acc[j + 3] += f.w;
            }
          }
        }
        uint32_t v[C::kChunk];
#pragma unroll
        for (int j = 0; j < C::kChunk; ++j) v[j] = __float_as_uint(acc[j]);
        store_chunk(v, c0);
      }
    }
    mes::cluster_sync();  // peers' partial tiles stay alive until every read is done
  }
  if (warp >= 2 && !C::kResidual) {
    if (lane == 0) mes::tma_store_wait_all<0>();
    __syncwarp();
  }

  mes::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    mes::tc_fence_after();
    mes::tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ----------------------------------------------------------------------------------------
// Persistent variant for large M.  One CTA per SM walks the (128-feature, BT-token) tiles
// in order (features fastest, so concurrently running CTAs share X rows in L2):
//   warp 0      TMA: X tile, packed weight words, and the group's scales/zero words of
//               every k-step into an SST-deep shared-memory ring;
//   warp 1      MMA issue into one of two TMEM accumulators (tile i+1's mainloop runs
//               while the epilogue drains tile i);
//   warps 2..   SETS sets of four dequant warps (one per TMEM lane quadrant); set g
//               dequantises the k-steps it with it % SETS == g, so SETS stages are in
//               flight at once and the tcgen05.st latency of one stage overlaps the
//               arithmetic of the next;
//   last 8      epilogue (two per lane quadrant, alternating token chunks).
// TMEM: accumulators at columns [0, BT) and [BT, 2BT), then an AST-deep ring of
// dequantised A slots (32 columns each).  The shared-memory ring is deeper than the TMEM
// ring so that TMA loads run far enough ahead of the MMA to hide their latency.
// AST == 0 keeps the dequantised A tile in shared memory instead (one 16 KB, 128-byte
// swizzled K-major tile per stage) and issues tcgen05.mma with both operands from shared
// memory; TMEM then holds only the two accumulators.
template <int BT, int SST, int AST, int EPI, int SETS>
struct PCfg {
  static constexpr bool kResidual = EPI == kEpiResidual, kSilu = EPI == kEpiSilu;
  static constexpr int kDqWarps = 4 * SETS;
  static constexpr int kEpiWarps = 8;  // two per TMEM lane quadrant, alternating chunks
  static constexpr int kThreads = (2 + kDqWarps + kEpiWarps) * 32;
  static constexpr int kXStage = BT * kBK * 2;
  static constexpr int kWBytes = (kBK / 8) * kBN * 4;  // 8 words x 128 features
  static constexpr int kSBytes = kBN * 2;               // fp16 scales of the group
  static constexpr int kZBytes = (kBN / 8) * 4;         // packed zero-points of the group
  static constexpr int kWStage = kWBytes + 256 + 128;   // words | scales (256 B) | zeros (64 B)
  static constexpr int kChunk = kResidual ? 16 : 32;
  static constexpr int kOutBuf = kChunk * 32 * 2;
  static constexpr int kASlots = AST == 0 ? SST : AST;
  static constexpr int kAStage = AST == 0 ? kBN * kBK * 2 : 0;  // A tile in shared memory
  static constexpr int kOffX = 0;
  static constexpr int kOffA = SST * kXStage;
  static constexpr int kOffW = kOffA + SST * kAStage;
  static constexpr int kOffOut = kOffW + SST * kWStage;
  static constexpr int kOffBar = kOffOut + (kResidual ? 0 : kEpiWarps * kOutBuf);
  static constexpr int kSmem = kOffBar + 512 + 1024;
  static constexpr int kTmemNeed = 2 * BT + AST * 32;
  static_assert(kSmem <= 232448, "shared memory budget");
  static_assert((2 * SST + 2 * kASlots + 5) * 8 + 8 <= 512, "barrier area");
  static_assert(kTmemNeed <= 512, "TMEM budget");
  static_assert(kSBytes == 256 && kZBytes == 64 && kWStage % 128 == 0, "stage layout");
  static_assert(BT % 16 == 0 && BT <= 256 && kXStage % 1024 == 0, "tile");
};

template <int BT, int SST, int AST, int EPI, int SETS>
__global__ void __launch_bounds__(PCfg<BT, SST, AST, EPI, SETS>::kThreads, 1)
awq_gemm_persistent_kernel(const __grid_constant__ CUtensorMap map_x,
                           const __grid_constant__ CUtensorMap map_w,
                           const __grid_constant__ CUtensorMap map_s,
                           const __grid_constant__ CUtensorMap map_z,
                           const __grid_constant__ CUtensorMap map_y,
                           const __nv_bfloat16* __restrict__ bias, float* __restrict__ R,
                           int64_t ldr, int M, int N, int K) {
  using C = PCfg<BT, SST, AST, EPI, SETS>;
  constexpr uint32_t kTmemCols = 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem + C::kOffX;
  uint8_t* as = smem + C::kOffA;
  uint8_t* wst = smem + C::kOffW;
  __nv_bfloat16* outbuf = reinterpret_cast<__nv_bfloat16*>(smem + C::kOffOut);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* full = bars;                      // [SST] TMA landed
  uint64_t* empty = bars + SST;               // [SST] MMAs of the stage done
  uint64_t* afull = bars + 2 * SST;           // [kASlots] dequantised A written
  uint64_t* aempty = afull + C::kASlots;      // [kASlots] MMAs reading the A slot done
  uint64_t* acc_full = aempty + C::kASlots;   // [2] accumulator complete
  uint64_t* acc_empty = acc_full + 2;         // [2] accumulator drained
  uint64_t* drain = acc_empty + 2;            // abort path: all issued MMAs completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);


  const int warp = mes::warp_id(), lane = mes::lane_id();
  const int nk = K / kBK;
  const int num_n = N / kBN;
  const int num_tiles = num_n * ((M + BT - 1) / BT);

  if (threadIdx.x == 0) {
    for (int s = 0; s < SST; ++s) {
      mes::mbar_init(&full[s], 1);
      mes::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < C::kASlots; ++a) {
      mes::mbar_init(&afull[a], 4);
      mes::mbar_init(&aempty[a], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mes::mbar_init(&acc_full[b], 1);
      mes::mbar_init(&acc_empty[b], C::kEpiWarps);
    }
    mes::mbar_init(drain, 1);
    *abort_flag = 0;
    mes::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    mes::tma_prefetch_desc(&map_x);
    mes::tma_prefetch_desc(&map_w);
    mes::tma_prefetch_desc(&map_s);
    mes::tma_prefetch_desc(&map_z);
    if (!C::kResidual) mes::tma_prefetch_desc(&map_y);
  }
  if (warp == 1) {
    __syncwarp();
    mes::tmem_alloc(tmem_slot, kTmemCols);
    mes::tmem_relinquish();
  }
  mes::tc_fence_before();
  __syncthreads();
  mes::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_a = tmem + 2 * BT;

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------------
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int n0 = (tile % num_n) * kBN, t0 = (tile / num_n) * BT;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % SST;
          if (it >= SST &&
              !mes::mbar_wait(&empty[s], ((it / SST) & 1) ^ 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          uint8_t* w = wst + s * C::kWStage;
          mes::mbar_arrive_expect_tx(&full[s], C::kXStage + C::kWBytes + C::kSBytes + C::kZBytes);
          mes::tma_load_2d(xs + s * C::kXStage, &map_x, &full[s], kb * kBK, t0);
          mes::tma_load_2d(w, &map_w, &full[s], n0, kb * (kBK / 8));
          mes::tma_load_2d(w + C::kWBytes, &map_s, &full[s], n0, kb / 2);
          mes::tma_load_2d(w + C::kWBytes + 256, &map_z, &full[s], n0 / 8, kb / 2);
        }
      }
      if (!ok) {
        // Let the copies already issued (the last SST iterations at most) land before the
        // CTA exits.
        const uint64_t tstart = mes::globaltimer_ns();
        for (int i = it - SST < 0 ? 0 : it - SST; i < it; ++i) {
          while (!mes::mbar_try_wait(&full[i % SST], (i / SST) & 1) &&
                 mes::globaltimer_ns() - tstart < mes::kWaitLimitNs) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------- MMA issuer ---------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = mes::idesc_bf16_f32(kBN, BT, false);
      const uint32_t xs_addr = mes::smem_u32(xs), as_addr = mes::smem_u32(as);
      int it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++lt) {
        const int b = lt & 1;
        if (lt >= 2 &&
            !mes::mbar_wait(&acc_empty[b], ((lt >> 1) - 1) & 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT)) {
          ok = false;
          break;
        }
        mes::tc_fence_after();
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % SST, a = it % C::kASlots;
          // afull implies full: every dequant warp waited for the whole stage (X included)
          // before arriving, so one barrier check per k-step suffices.
          if (!mes::mbar_wait(&afull[a], (it / C::kASlots) & 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          mes::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t bdesc = mes::smem_desc_sw128(xs_addr + s * C::kXStage + kk * 32, 16, 1024);
            if constexpr (AST == 0) {
              const uint64_t adesc = mes::smem_desc_sw128(as_addr + s * C::kAStage + kk * 32, 16, 1024);
              mes::mma_ss(tmem + b * BT, adesc, bdesc, idesc, (kb | kk) != 0);
            } else {
              mes::mma_ts(tmem + b * BT, tmem_a + a * 32 + kk * 8, bdesc, idesc, (kb | kk) != 0);
            }
          }
          mes::tc_commit(&empty[s]);
          if constexpr (AST != 0) mes::tc_commit(&aempty[a]);
        }
        mes::tc_commit(&acc_full[b]);
      }
      if (!ok) {
        // Wait (bounded) until every MMA issued so far has completed.
        mes::tc_commit(drain);
        const uint64_t tstart = mes::globaltimer_ns();
        while (!mes::mbar_try_wait(drain, 0) && mes::globaltimer_ns() - tstart < mes::kWaitLimitNs) {
        }
      }
    }
    __syncwarp();
  } else if (warp < 2 + C::kDqWarps) {
    // --------------------------------- dequant ----------------------------------------
    const int q = warp & 3;
    const int set = (warp - 2) / 4;
    const int row = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int zshift = 4 * kInvOrder[row & 7];  // n0 is a multiple of 128
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < nk; ++kb, ++it) {
        if (it % SETS != set) continue;
        const int s = it % SST, a = it % C::kASlots;
        // With A in shared memory the stage's own ring protects it (the producer refills
        // a stage only after its MMAs completed); with A in TMEM its slot is waited for.
        if (!mes::mbar_wait_warp(&full[s], (it / SST) & 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT) ||
            (AST != 0 && it >= AST &&
             !mes::mbar_wait_warp(&aempty[a], ((it / C::kASlots) & 1) ^ 1, abort_flag,
                                  &g_err_gemm, MES_ERR_TIMEOUT))) {
          ok = false;
          break;
        }
        mes::tc_fence_after();
        const uint8_t* w = wst + s * C::kWStage;
        const GroupParams gp =
            make_group(reinterpret_cast<const uint32_t*>(w + C::kWBytes + 256)[row >> 3], zshift,
                       reinterpret_cast<const uint16_t*>(w + C::kWBytes)[row]);
        const uint32_t* wsrc = reinterpret_cast<const uint32_t*>(w) + row;
        uint32_t av[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t v = wsrc[i * kBN];
          av[4 * i + 0] = dq_pair(v, gp);
          av[4 * i + 1] = dq_pair(v >> 4, gp);
          av[4 * i + 2] = dq_pair(v >> 8, gp);
          av[4 * i + 3] = dq_pair(v >> 12, gp);
        }
        if constexpr (AST == 0) {
          // Row `row` of the 128 x 64 K-major tile, 128-byte swizzle: 16-byte chunk i
          // (k = 8i .. 8i+7) lives at chunk position i ^ (row & 7).
          uint8_t* arow = as + s * C::kAStage + row * 128;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<uint4*>(arow + ((i ^ (row & 7)) * 16)) =
                make_uint4(av[4 * i], av[4 * i + 1], av[4 * i + 2], av[4 * i + 3]);
          mes::fence_proxy_async_smem();
        } else {
          mes::tmem_st32(tmem_a + a * 32 + lane_off, av);
          mes::tmem_wait_st();
        }
        mes::tc_fence_before();
        __syncwarp();
        if (lane == 0) mes::mbar_arrive(&afull[a]);
        __syncwarp();
      }
    }
  } else {
    // --------------------------------- epilogue ---------------------------------------
    const int q = warp & 3;
    const int eh = (warp - 2 - C::kDqWarps) / 4;  // which alternate chunks this warp drains
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    __nv_bfloat16* buf = outbuf + (warp - 2 - C::kDqWarps) * (C::kOutBuf / 2);
    bool stored = false;
    int lt = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++lt) {
      const int b = lt & 1;
      const int n0 = (tile % num_n) * kBN, t0 = (tile / num_n) * BT;
      const int n = n0 + q * 32 + lane;
      if (!mes::mbar_wait_warp(&acc_full[b], (lt >> 1) & 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT))
        break;
      mes::tc_fence_after();
      const float bv = bias ? __bfloat162float(bias[n]) : 0.f;
#pragma unroll 1
      for (int c0 = eh * C::kChunk; c0 < BT; c0 += 2 * C::kChunk) {
        uint32_t v[C::kChunk];
        if constexpr (C::kChunk == 32) mes::tmem_ld32(tmem + lane_off + b * BT + c0, v);
        else mes::tmem_ld16(tmem + lane_off + b * BT + c0, v);
        mes::tmem_wait_ld();
        if (t0 + c0 >= M) continue;  // rows past the end of X
        if constexpr (C::kSilu) {
          silu_chunk<C::kChunk>(v, lane, buf, stored, &map_y, n0 / 2 + q * 16, t0 + c0);
        } else if constexpr (C::kResidual) {
          const int rows = min(C::kChunk, M - (t0 + c0));
          float* rp = R + (int64_t)(t0 + c0) * ldr + n;
          float rv[C::kChunk];
#pragma unroll
          for (int j = 0; j < C::kChunk; ++j) rv[j] = j < rows ? rp[(int64_t)j * ldr] : 0.f;
#pragma unroll
          for (int j = 0; j < C::kChunk; ++j)
            if (j < rows) rp[(int64_t)j * ldr] = rv[j] + (__uint_as_float(v[j]) + bv);
        } else {
          if (stored) {
            if (lane == 0) mes::tma_store_wait_read<0>();
            __syncwarp();
          }
#pragma unroll
          for (int j = 0; j < C::kChunk; j += 2) {  // one bf16x2 conversion per two values
            const uint32_t pk = mes::pack_bf16x2(__uint_as_float(v[j]) + bv, __uint_as_float(v[j + 1]) + bv);
            buf[j * 32 + lane] = __ushort_as_bfloat16(static_cast<unsigned short>(pk & 0xFFFFu));
            buf[(j + 1) * 32 + lane] = __ushort_as_bfloat16(static_cast<unsigned short>(pk >> 16));
          }
          mes::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mes::tma_store_2d(&map_y, buf, n0 + q * 32, t0 + c0);
            mes::tma_store_commit();
          }
          __syncwarp();
          stored = true;
        }
      }
      // The accumulator is free once every tcgen05.ld above has completed.
      mes::tc_fence_before();
      __syncwarp();
      if (lane == 0) mes::mbar_arrive(&acc_empty[b]);
      __syncwarp();
    }
    if (!C::kResidual) {
      if (lane == 0) mes::tma_store_wait_all<0>();
      __syncwarp();
    }
  }

  mes::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    mes::tc_fence_after();
    mes::tmem_dealloc(tmem, kTmemCols);
  }
}

// ----------------------------------------------------------------------------------------
// Pair variant (clusters of two CTAs on neighbouring SMs, tcgen05 cta_group::2).  A pair
// computes a 256-feature x 256-token tile: CTA r holds features [128r, 128r + 128) of the
// tile as A and tokens [128r, 128r + 128) of X as B; one MMA of M = 256, N = 256 in the
// even CTA reads A's rows and B's rows from both CTAs' shared memory and leaves each CTA's
// 128 features x 256 tokens in that CTA's TMEM.  Against the single-CTA kernel every SM
// stages and reads half the X bytes per k-step (tensor-core operand reads 32 KB instead of
// 48 KB), which lowers the shared-memory traffic that bounds the single-CTA mainloop.
//
// Two ways to fill A (PANEL):
//   false  dequant warps (SETS sets of four) turn the stage's packed weight words, scales
//          and zeros (TMA-loaded per CTA) into the 128 x 64 A tile, as in the single-CTA
//          kernel;
//   true   A is TMA-loaded from a bf16 weight panel W^T [N, K] that awq_panel_kernel
//          dequantised just before (same exact arithmetic).  No dequant warps: the
//          mainloop is the tensor pipe and TMA alone, and the panel (N*K*2 bytes) is read
//          from L2.
// Roles per CTA: warp 0 TMA producer, warp 1 MMA issuer (even CTA only; the odd CTA's
// warp 1 only takes part in the TMEM allocation), [dequant warps], 8 epilogue warps.
// Barriers:
//   full_x[s]  (even CTA)  both X halves landed (PANEL: both X and both A halves):
//                          expect_tx by the even producer, complete_tx from both CTAs'
//                          loads.  Fused: waited for by the even CTA's dequant warps, so
//                          the MMA's wait on afull covers it; PANEL: waited for by the MMA;
//   full_w[s]  (each CTA)  fused only: the CTA's weight words, scales and zeros landed;
//   afull[s]   (even CTA)  fused only: A rows of both CTAs written (4 dequant warps of
//                          each CTA arrive per set);
//   empty[s]   (each CTA)  the stage's MMAs done (commit multicast to both CTAs);
//   acc_full[b] (each CTA) accumulator b complete (commit multicast);
//   acc_empty[b] (even CTA) accumulator b drained in both CTAs (8 epilogue warps each);
//   drain      (each CTA)  abort path only: every MMA issued so far has completed.
// Tile order (pair_tile): feature tiles are grouped into bands of `band` tiles; the pairs
// walk one band at a time, features fastest inside it.  A band's panel rows stay in L2
// while every token tile passes them, and the X tiles of a token row are shared by the
// pairs working on that row at the same time.
template <int EPI, bool PANEL>
struct QCfg {
  static constexpr bool kResidual = EPI == kEpiResidual, kSilu = EPI == kEpiSilu;
  static constexpr int SETS = PANEL ? 0 : 2;
  // The panel variant's stages have no weight words, which leaves room for one more stage.
  static constexpr int SST = PANEL ? 6 : 5;
  static constexpr int kDqWarps = 4 * SETS;
  static constexpr int kEpiWarps = 8;
  static constexpr int kThreads = (2 + kDqWarps + kEpiWarps) * 32;
  static constexpr int kTileN = 2 * kBN;   // features per pair tile
  static constexpr int kTileT = 256;       // tokens per pair tile
  static constexpr int kHalfT = kTileT / 2;
  static constexpr int kXStage = kHalfT * kBK * 2;
  static constexpr int kAStage = kBN * kBK * 2;
  static constexpr int kWBytes = PANEL ? 0 : (kBK / 8) * kBN * 4;
  static constexpr int kSBytes = kBN * 2;
  static constexpr int kZBytes = (kBN / 8) * 4;
  static constexpr int kWStage = PANEL ? 0 : kWBytes + 256 + 128;
  static constexpr int kChunk = kResidual ? 16 : 32;
  // Staging per epilogue warp: a 32-feature x 32-token bf16 block, or two 32 x 16 fp32
  // blocks for the residual's TMA reduce-add (one filling while the other is read).
  static constexpr int kOutBuf = kResidual ? 2 * kChunk * 32 * 4 : kChunk * 32 * 2;
  static constexpr int kOffX = 0;
  static constexpr int kOffA = SST * kXStage;
  static constexpr int kOffW = kOffA + SST * kAStage;
  static constexpr int kOffOut = kOffW + SST * kWStage;
  static constexpr int kOffBar = kOffOut + kEpiWarps * kOutBuf;
  static constexpr int kSmem = kOffBar + 512 + 1024;
  static_assert(kSmem <= 232448, "shared memory budget");
  static_assert((4 * SST + 5) * 8 + 8 <= 512, "barrier area");
  static_assert(kSBytes == 256 && kZBytes == 64 && kWStage % 128 == 0, "stage layout");
  static_assert(kXStage % 1024 == 0 && kAStage % 1024 == 0, "swizzle atoms");
};

// (feature tile, token tile) of pair tile `tile` in the banded order described above.
__device__ __forceinline__ void pair_tile(int tile, int num_n, int num_t, int band, int& f,
                                          int& t) {
  const int per_band = band * num_t;
  const int b = tile / per_band, r = tile - b * per_band;
  const int width = min(band, num_n - b * band);
  f = b * band + r % width;
  t = r / width;
}

// Work item `i` of the pair kernels: the first `full` items are whole 256-token tiles in the
// banded order; when the tiles leave a last round that would occupy at most half of the
// pairs, the host makes the remaining tiles into two 128-token halves each (items `full`,
// `full` + 1, ...), so the last round takes half a tile's time on twice as many pairs.
struct PairItem {
  int f;     // feature tile (256 features)
  int t0;    // first token
  int ntok;  // 256, or 128 for a half tile
};
__device__ __forceinline__ PairItem pair_item(int i, int full, int num_n, int num_t, int band) {
  PairItem p;
  const int tile = i < full ? i : full + ((i - full) >> 1);
  int t;
  pair_tile(tile, num_n, num_t, band, p.f, t);
  p.ntok = i < full ? 256 : 128;
  p.t0 = t * 256 + (i < full ? 0 : ((i - full) & 1) * 128);
  return p;
}

template <int EPI, bool PANEL>
__global__ void __launch_bounds__(QCfg<EPI, PANEL>::kThreads, 1)
awq_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_x,
                     const __grid_constant__ CUtensorMap map_w,
                     const __grid_constant__ CUtensorMap map_s,
                     const __grid_constant__ CUtensorMap map_z,
                     const __grid_constant__ CUtensorMap map_y,
                     const __nv_bfloat16* __restrict__ bias, float* __restrict__ R, int64_t ldr,
                     int M, int N, int K, int band, int full, int num_items, int res_tma) {
  using C = QCfg<EPI, PANEL>;
  constexpr int SST = C::SST;
  constexpr uint32_t kTmemCols = 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem + C::kOffX;
  uint8_t* as = smem + C::kOffA;
  uint8_t* wst = smem + C::kOffW;
  __nv_bfloat16* outbuf = reinterpret_cast<__nv_bfloat16*>(smem + C::kOffOut);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* full_x = bars;              // [SST]
  uint64_t* full_w = bars + SST;        // [SST]
  uint64_t* afull = bars + 2 * SST;     // [SST]
  uint64_t* empty = bars + 3 * SST;     // [SST]
  uint64_t* acc_full = bars + 4 * SST;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* drain = acc_empty + 2;      // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = mes::warp_id(), lane = mes::lane_id();
  const uint32_t rank = mes::cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int nk = K / kBK;
  const int num_n = N / C::kTileN;
  const int num_t = (M + C::kTileT - 1) / C::kTileT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SST; ++s) {
      mes::mbar_init(&full_x[s], 1);
      mes::mbar_init(&full_w[s], 1);
      mes::mbar_init(&afull[s], 8);
      mes::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mes::mbar_init(&acc_full[b], 1);
      mes::mbar_init(&acc_empty[b], 2 * C::kEpiWarps);
    }
    mes::mbar_init(drain, 1);
    *abort_flag = 0;
    mes::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    mes::tma_prefetch_desc(&map_x);
    mes::tma_prefetch_desc(&map_w);
    if constexpr (!PANEL) {
      mes::tma_prefetch_desc(&map_s);
      mes::tma_prefetch_desc(&map_z);
    }
    if (EPI != kEpiResidual || res_tma) mes::tma_prefetch_desc(&map_y);
  }
  if (warp == 1) {
    __syncwarp();
    mes::tmem_alloc2(tmem_slot, kTmemCols);
    mes::tmem_relinquish2();
  }
  mes::tc_fence_before();
  mes::cluster_sync();  // both CTAs' barriers are initialised before either signals the other
  mes::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------------
    if (lane == 0) {
      const uint32_t full_x0 = mes::mapa_shared(mes::smem_u32(full_x), 0);
      int it = 0;
      bool ok = true;
      for (int item = pair; item < num_items && ok; item += npairs) {
        // A half tile uses the first 64 rows of each CTA's 128-row X box.
        const PairItem pi = pair_item(item, full, num_n, num_t, band);
        const int n0 = pi.f * C::kTileN + (int)rank * kBN;
        const int t0 = pi.t0 + (int)rank * (pi.ntok / 2);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % SST;
          if (it >= SST &&
              !mes::mbar_wait(&empty[s], ((it / SST) & 1) ^ 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          if constexpr (PANEL) {
            if (rank == 0) mes::mbar_arrive_expect_tx(&full_x[s], 2 * (C::kXStage + C::kAStage));
            mes::tma_load_2d_pair(as + s * C::kAStage, &map_w, full_x0 + 8 * s, kb * kBK, n0);
            mes::tma_load_2d_pair(xs + s * C::kXStage, &map_x, full_x0 + 8 * s, kb * kBK, t0);
          } else {
            if (rank == 0) mes::mbar_arrive_expect_tx(&full_x[s], 2 * C::kXStage);
            mes::tma_load_2d_pair(xs + s * C::kXStage, &map_x, full_x0 + 8 * s, kb * kBK, t0);
            uint8_t* w = wst + s * C::kWStage;
            mes::mbar_arrive_expect_tx(&full_w[s], C::kWBytes + C::kSBytes + C::kZBytes);
            mes::tma_load_2d(w, &map_w, &full_w[s], n0, kb * (kBK / 8));
            mes::tma_load_2d(w + C::kWBytes, &map_s, &full_w[s], n0, kb / 2);
            mes::tma_load_2d(w + C::kWBytes + 256, &map_z, &full_w[s], n0 / 8, kb / 2);
          }
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA exits: the even CTA's full_x
        // counts both CTAs' pair copies of every stage it armed, full_w this CTA's own
        // copies.  (The cluster barrier at the end keeps the odd CTA until then.)
        const uint64_t tstart = mes::globaltimer_ns();
        for (int i = it - SST < 0 ? 0 : it - SST; i < it; ++i) {
          while (((rank == 0 && !mes::mbar_try_wait(&full_x[i % SST], (i / SST) & 1)) ||
                  (!PANEL && !mes::mbar_try_wait(&full_w[i % SST], (i / SST) & 1))) &&
                 mes::globaltimer_ns() - tstart < mes::kWaitLimitNs) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------- MMA issuer (even CTA) ----------------------------
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc_full = mes::idesc_bf16_f32(2 * kBN, C::kTileT, false);
      constexpr uint32_t idesc_half = mes::idesc_bf16_f32(2 * kBN, C::kTileT / 2, false);
      const uint32_t xs_addr = mes::smem_u32(xs), as_addr = mes::smem_u32(as);
      int it = 0, lt = 0;
      bool ok = true;
      for (int item = pair; item < num_items && ok; item += npairs, ++lt) {
        const uint32_t idesc = item < full ? idesc_full : idesc_half;
        const int b = lt & 1;
        if (lt >= 2 &&
            !mes::mbar_wait(&acc_empty[b], ((lt >> 1) - 1) & 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT)) {
          ok = false;
          break;
        }
        mes::tc_fence_after();
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % SST;
          // Fused: afull implies full_x (the even CTA's dequant warps wait for both X halves
          // before arriving), so one barrier check per k-step suffices.
          uint64_t* ready = PANEL ? &full_x[s] : &afull[s];
          if (!mes::mbar_wait(ready, (it / SST) & 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          mes::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t adesc = mes::smem_desc_sw128(as_addr + s * C::kAStage + kk * 32, 16, 1024);
            const uint64_t bdesc = mes::smem_desc_sw128(xs_addr + s * C::kXStage + kk * 32, 16, 1024);
            mes::mma_ss2(tmem + b * C::kTileT, adesc, bdesc, idesc, (kb | kk) != 0);
          }
          mes::tc_commit2_mc(&empty[s], 0x3);
        }
        if (ok) mes::tc_commit2_mc(&acc_full[b], 0x3);
      }
      if (!ok) {
        // Wait (bounded) until every MMA issued so far has completed.
        mes::tc_commit2_mc(drain, 0x1);
        const uint64_t tstart = mes::globaltimer_ns();
        while (!mes::mbar_try_wait(drain, 0) && mes::globaltimer_ns() - tstart < mes::kWaitLimitNs) {
        }
      }
    }
    __syncwarp();
  } else if (warp < 2 + C::kDqWarps) {
    // --------------------------------- dequant (fused only) ---------------------------
    if constexpr (!PANEL) {
      const int set = (warp - 2) / 4;
      const int row = (warp & 3) * 32 + lane;
      const int zshift = 4 * kInvOrder[row & 7];  // n0 is a multiple of 128
      const uint32_t afull0 = mes::mapa_shared(mes::smem_u32(afull), 0);
      int it = 0;
      bool ok = true;
      for (int item = pair; item < num_items && ok; item += npairs) {
        for (int kb = 0; kb < nk; ++kb, ++it) {
          if (it % C::SETS != set) continue;
          const int s = it % SST;
          // The A slot of a stage is free once the stage's weights landed again: the
          // producer refills a stage only after its MMAs completed.
          if (!mes::mbar_wait_warp(&full_w[s], (it / SST) & 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT) ||
              (rank == 0 &&
               !mes::mbar_wait_warp(&full_x[s], (it / SST) & 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT))) {
            ok = false;
            break;
          }
          const uint8_t* w = wst + s * C::kWStage;
          const GroupParams gp =
              make_group(reinterpret_cast<const uint32_t*>(w + C::kWBytes + 256)[row >> 3], zshift,
                         reinterpret_cast<const uint16_t*>(w + C::kWBytes)[row]);
          const uint32_t* wsrc = reinterpret_cast<const uint32_t*>(w) + row;
          uint32_t av[32];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t v = wsrc[i * kBN];
            av[4 * i + 0] = dq_pair(v, gp);
            av[4 * i + 1] = dq_pair(v >> 4, gp);
            av[4 * i + 2] = dq_pair(v >> 8, gp);
            av[4 * i + 3] = dq_pair(v >> 12, gp);
          }
          // Row `row` of the 128 x 64 K-major tile, 128-byte swizzle: 16-byte chunk i
          // (k = 8i .. 8i+7) lives at chunk position i ^ (row & 7).
          uint8_t* arow = as + s * C::kAStage + row * 128;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<uint4*>(arow + ((i ^ (row & 7)) * 16)) =
                make_uint4(av[4 * i], av[4 * i + 1], av[4 * i + 2], av[4 * i + 3]);
          mes::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mes::mbar_arrive_remote(afull0 + 8 * s);
          __syncwarp();
        }
      }
    }
  } else {
    // --------------------------------- epilogue ---------------------------------------
    const int q = warp & 3;
    const int eh = (warp - 2 - C::kDqWarps) / 4;  // which alternate chunks this warp drains
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t acc_empty0 = mes::mapa_shared(mes::smem_u32(acc_empty), 0);
    __nv_bfloat16* buf = outbuf + (warp - 2 - C::kDqWarps) * (C::kOutBuf / 2);
    bool stored = false;
    int nchunk = 0;  // residual chunks handed to TMA reduce-adds by this warp
    int lt = 0;
    for (int item = pair; item < num_items; item += npairs, ++lt) {
      const int b = lt & 1;
      const PairItem pi = pair_item(item, full, num_n, num_t, band);
      const int n0 = pi.f * C::kTileN + (int)rank * kBN;
      const int t0 = pi.t0;
      const int n = n0 + q * 32 + lane;
      if (!mes::mbar_wait_warp(&acc_full[b], (lt >> 1) & 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT))
        break;
      mes::tc_fence_after();
      const float bv = bias ? __bfloat162float(bias[n]) : 0.f;
#pragma unroll 1
      for (int c0 = eh * C::kChunk; c0 < pi.ntok; c0 += 2 * C::kChunk) {
        uint32_t v[C::kChunk];
        if constexpr (C::kChunk == 32) mes::tmem_ld32(tmem + lane_off + b * C::kTileT + c0, v);
        else mes::tmem_ld16(tmem + lane_off + b * C::kTileT + c0, v);
        mes::tmem_wait_ld();
        if (t0 + c0 >= M) continue;  // rows past the end of X
        if constexpr (C::kSilu) {
          silu_chunk<C::kChunk>(v, lane, buf, stored, &map_y, n0 / 2 + q * 16, t0 + c0);
        } else if constexpr (C::kResidual) {
          if (res_tma) {
            // acc + bias goes to a staging block; a TMA reduce-add adds it into R in L2, so
            // the epilogue never waits on R's loads.  Each element of R gets one fp32 add
            // (R + (acc + bias), rounded once), as in the register path below.  Rows past M
            // are clipped by the tensor map.
            float* stg = reinterpret_cast<float*>(buf) + (nchunk & 1) * (C::kChunk * 32);
            if (nchunk >= 2) {  // the reduce that last read this block must be done reading
              if (lane == 0) mes::tma_store_wait_read<1>();
              __syncwarp();
            }
#pragma unroll
            for (int j = 0; j < C::kChunk; ++j) stg[j * 32 + lane] = __uint_as_float(v[j]) + bv;
            mes::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              mes::tma_reduce_add_2d(&map_y, stg, n0 + q * 32, t0 + c0);
              mes::tma_store_commit();
            }
            __syncwarp();
            ++nchunk;
          } else {
            const int rows = min(C::kChunk, M - (t0 + c0));
            float* rp = R + (int64_t)(t0 + c0) * ldr + n;
            float rv[C::kChunk];
#pragma unroll
            for (int j = 0; j < C::kChunk; ++j) rv[j] = j < rows ? rp[(int64_t)j * ldr] : 0.f;
#pragma unroll
            for (int j = 0; j < C::kChunk; ++j)
              if (j < rows) rp[(int64_t)j * ldr] = rv[j] + (__uint_as_float(v[j]) + bv);
          }
        } else {
          if (stored) {
            if (lane == 0) mes::tma_store_wait_read<0>();
            __syncwarp();
          }
#pragma unroll
          for (int j = 0; j < C::kChunk; j += 2) {  // one bf16x2 conversion per two values
            const uint32_t pk = mes::pack_bf16x2(__uint_as_float(v[j]) + bv, __uint_as_float(v[j + 1]) + bv);
            buf[j * 32 + lane] = __ushort_as_bfloat16(static_cast<unsigned short>(pk & 0xFFFFu));
            buf[(j + 1) * 32 + lane] = __ushort_as_bfloat16(static_cast<unsigned short>(pk >> 16));
          }
          mes::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mes::tma_store_2d(&map_y, buf, n0 + q * 32, t0 + c0);
            mes::tma_store_commit();
          }
          __syncwarp();
          stored = true;
        }
      }
      // The accumulator is free once every tcgen05.ld above has completed, in both CTAs.
      mes::tc_fence_before();
      __syncwarp();
      if (lane == 0) mes::mbar_arrive_remote(acc_empty0 + 8 * b);
      __syncwarp();
    }
    if (lane == 0) mes::tma_store_wait_all<0>();  // stores / reduce-adds complete
    __syncwarp();
  }

  mes::tc_fence_before();
  __syncthreads();
  mes::cluster_sync();  // no signal of either CTA can reach a CTA that has left
  if (warp == 1) {
    __syncwarp();
    mes::tc_fence_after();
    mes::tmem_dealloc2(tmem, kTmemCols);
  }
}

// ------------------------------------ weight panel ----------------------------------------
// W^T [N, K] bf16 (K contiguous) from the kernel-layout AWQ tensors, with the GEMM's exact
// dequantisation: the A operand of the PANEL pair kernel.  One launch builds up to
// kMaxPanels panels (the projections of one decoder layer).  A block of 256 threads covers
// 8 features x 32 words (256 k) of one panel: warp f takes feature n0 + f, lane b word
// b0 + b, so a warp writes 512 contiguous bytes of its feature's row, and the eight warps
// read the same 32 sectors of the packed words (one per word row, eight features each)
// through L1.
constexpr int kMaxPanels = 8;
struct PanelJob {
  const uint32_t* qw;
  const int32_t* qzeros;
  const uint16_t* scales;
  uint4* out;
  int K, N;
  int kblocks;      // blocks along K: ceil(K / 8 / 32)
  int first_block;  // first block index of this panel in the launch
};
struct PanelJobs {
  PanelJob job[kMaxPanels];
  int count;
};

__global__ void __launch_bounds__(256) awq_panel_kernel(const __grid_constant__ PanelJobs jobs) {
  int p = 0;
  while (p + 1 < jobs.count && (int)blockIdx.x >= jobs.job[p + 1].first_block) ++p;
  const PanelJob& jb = jobs.job[p];
  const int local = blockIdx.x - jb.first_block;
  const int f = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = (local / jb.kblocks) * 8 + f;
  const int b = (local % jb.kblocks) * 32 + lane;
  if (b >= jb.K / 8) return;
  const int N = jb.N;
  const int g = (8 * b) / kGroup;
  const GroupParams gp = make_group(__ldg(jb.qzeros + (int64_t)g * (N / 8) + (n >> 3)),
                                    4 * kInvOrder[n & 7], __ldg(jb.scales + (int64_t)g * N + n));
  const uint32_t w = __ldg(jb.qw + (int64_t)b * N + n);
  uint4 v;
  v.x = dq_pair(w, gp);
  v.y = dq_pair(w >> 4, gp);
  v.z = dq_pair(w >> 8, gp);
  v.w = dq_pair(w >> 12, gp);
  jb.out[(int64_t)n * (jb.K / 8) + b] = v;
}

// ------------------------------------ repack ----------------------------------------------
// out[b, n] = sum_i code(k = 8b + order[i], n) << 4i, order = {0,2,4,6,1,3,5,7}.
__global__ void awq_repack_kernel(const uint32_t* __restrict__ in, int64_t K, int64_t N,
                                  uint32_t* __restrict__ out) {
  const int64_t total = (K / 8) * N;
  const int order[8] = {0, 2, 4, 6, 1, 3, 5, 7};
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / N, n = i - b * N;
    const int sh = 4 * kInvOrder[n & 7];
    uint32_t w = 0;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const uint32_t src = __ldg(in + (8 * b + order[p]) * (N / 8) + (n >> 3));
      w |= ((src >> sh) & 0xFu) << (4 * p);
    }
    out[i] = w;
  }
}

// ------------------------------------ dequant ---------------------------------------------
// One thread per (feature n, word b): writes W^T[n, 8b .. 8b+7] (16 bytes).
__global__ void awq_dequant_kernel(const uint32_t* __restrict__ qw, const int32_t* __restrict__ qzeros,
                                   const uint16_t* __restrict__ scales, int64_t K, int64_t N,
                                   uint4* __restrict__ out) {
  const int64_t total = (K / 8) * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / (K / 8), b = i - n * (K / 8);
    const int64_t g = (8 * b) / kGroup;
    const GroupParams gp = make_group(__ldg(qzeros + g * (N / 8) + (n >> 3)),
                                      4 * kInvOrder[n & 7], __ldg(scales + g * N + n));
    const uint32_t w = __ldg(qw + b * N + n);
    uint4 v;
    v.x = dq_pair(w, gp);
    v.y = dq_pair(w >> 4, gp);
    v.z = dq_pair(w >> 8, gp);
    v.w = dq_pair(w >> 12, gp);
    out[n * (K / 8) + b] = v;
  }
}

// Output tensor map of an epilogue mode: bf16 Y [M, N], or Y [M, N/2] for SiLU-and-mul.
inline bool make_out_map(CUtensorMap* my, const CUtensorMap& fallback, int epi, void* Y, int64_t M,
                         int64_t N, int64_t ldy, int chunk) {
  if (epi == kEpiResidual) {
    *my = fallback;  // unused by the residual epilogue
    return true;
  }
  const int64_t cols = epi == kEpiSilu ? N / 2 : N;
  return mes_host::make_map_2d(my, Y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, cols, ldy, chunk,
                               epi == kEpiSilu ? 16 : 32, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Number of CTAs that share the K range of one tile (small-M kernel): enough for one CTA
// per SM outside the reserve, at most 8 (a portable cluster) and at most the K / 128 weight
// groups; reduced until the clusters of one wave fit on the device at once.  The
// environment variable MES_GEMM_SPLIT (read once) fixes it for tuning; 0 or unset = auto.
// `clusters_by` caches the resident-cluster count per device and split size for `kern`.
template <typename Kern>
int choose_split(Kern kern, cudaLaunchConfig_t cfg, int64_t tiles, int64_t groups,
                 std::atomic<int> (&clusters_by)[64][9]) {
  static const int forced = [] {
    const char* v = getenv("MES_GEMM_SPLIT");
    const int c = v ? atoi(v) : 0;
    return (c < 0 || c > 8) ? 0 : c;
  }();
  const int sms = mes_host::persistent_ctas();
  int split = forced > 0 ? forced : (tiles >= sms ? 1 : (int)(sms / tiles));
  if (split > 8) split = 8;
  if (split > groups) split = (int)groups;
  if (forced > 0 || split <= 1) return split < 1 ? 1 : split;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 1;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  for (; split > 1; --split) {
    int clusters = clusters_by[dev & 63][split].load(std::memory_order_relaxed);
    if (clusters == 0) {
      attr[0].val.clusterDim.x = split;
      cfg.gridDim = dim3((unsigned)split, 1, 1);
      if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        clusters = 0;
      }
      if (clusters <= 0) clusters = -1;
      clusters_by[dev & 63][split].store(clusters, std::memory_order_relaxed);
    }
    if (clusters >= tiles) break;
  }
  return split;
}

// One-tile-per-CTA launch (split-K over clusters when the tile grid leaves SMs idle).
template <int BT, int STAGES, int ASLOTS, int EPI, int NDQ>
int launch_gemm(const void* X, int64_t ldx, const int32_t* qw, const int32_t* qzeros,
                const void* scales, const void* bias, void* Y, int64_t ldy, int64_t M,
                int64_t N, int64_t K, cudaStream_t stream) {
  using C = Cfg<BT, STAGES, ASLOTS, EPI, NDQ>;
  auto kern = awq_gemm_kernel<BT, STAGES, ASLOTS, EPI, NDQ>;
  static std::atomic<uint64_t> attr_done{0};
  const int st = mes_host::once_per_device(attr_done, [&] {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemLaunch) !=
        cudaSuccess)
      return MES_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, C::kThreads, C::kSmemLaunch) !=
            cudaSuccess ||
        per_sm < 1 || per_sm > C::kCtasByTmem)
      return MES_ERR_CUDA;  // more CTAs per SM than TMEM serves: refuse rather than risk a wait
    return MES_OK;
  });
  if (st != MES_OK) return st;
  CUtensorMap mx, mw, ms, mz, my;
  if (!mes_host::make_map_2d(&mx, X, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, ldx, BT, kBK,
                             CU_TENSOR_MAP_SWIZZLE_128B) ||
      !mes_host::make_map_2d(&mw, qw, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, K / 8, N, N, kBK / 8, kBN,
                             CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !mes_host::make_map_2d(&ms, scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, K / kGroup, N, N, 1,
                             kBN, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !mes_host::make_map_2d(&mz, qzeros, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, K / kGroup, N / 8,
                             N / 8, 1, kBN / 8, CU_TENSOR_MAP_SWIZZLE_NONE))
    return MES_ERR_INVALID;
  if (!make_out_map(&my, mx, EPI, Y, M, N, ldy, C::kChunk)) return MES_ERR_INVALID;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemLaunch;
  cfg.stream = stream;
  const int64_t tiles = (N / kBN) * ((M + BT - 1) / BT);
  static std::atomic<int> clusters_by[64][9];  // resident clusters, per device and split
  const int split = choose_split(kern, cfg, tiles, K / kGroup, clusters_by);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = split > 1 ? 1 : 0;
  cfg.gridDim = dim3((unsigned)(N / kBN * split), (unsigned)((M + BT - 1) / BT), 1);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mx, mw, ms, mz, my, (const __nv_bfloat16*)bias,
                                           C::kResidual ? (float*)Y : nullptr, ldy, (int)M, (int)N,
                                           (int)K, split);
  if (e != cudaSuccess) return MES_ERR_CUDA;
  return mes_host::from_cuda(cudaGetLastError());
}

template <int BT, int SST, int AST, int EPI, int SETS>
int launch_gemm_persistent(const void* X, int64_t ldx, const int32_t* qw, const int32_t* qzeros,
                           const void* scales, const void* bias, void* Y, int64_t ldy, int64_t M,
                           int64_t N, int64_t K, cudaStream_t stream) {
  using C = PCfg<BT, SST, AST, EPI, SETS>;
  static std::atomic<uint64_t> attr_done{0};
  const int st = mes_host::once_per_device(attr_done, [] {
    return cudaFuncSetAttribute(awq_gemm_persistent_kernel<BT, SST, AST, EPI, SETS>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) == cudaSuccess
               ? MES_OK : MES_ERR_CUDA;
  });
  if (st != MES_OK) return st;
  CUtensorMap mx, mw, ms, mz, my;
  if (!mes_host::make_map_2d(&mx, X, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, ldx, BT, kBK,
                             CU_TENSOR_MAP_SWIZZLE_128B) ||
      !mes_host::make_map_2d(&mw, qw, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, K / 8, N, N, kBK / 8, kBN,
                             CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !mes_host::make_map_2d(&ms, scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, K / kGroup, N, N, 1,
                             kBN, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !mes_host::make_map_2d(&mz, qzeros, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, K / kGroup, N / 8,
                             N / 8, 1, kBN / 8, CU_TENSOR_MAP_SWIZZLE_NONE))
    return MES_ERR_INVALID;
  if (!make_out_map(&my, mx, EPI, Y, M, N, ldy, C::kChunk)) return MES_ERR_INVALID;
  const int64_t tiles = (N / kBN) * ((M + BT - 1) / BT);
  const int ctas = mes_host::persistent_ctas();
  const int grid = (int)(tiles < ctas ? tiles : ctas);
  awq_gemm_persistent_kernel<BT, SST, AST, EPI, SETS><<<grid, C::kThreads, C::kSmem, stream>>>(
      mx, mw, ms, mz, my, (const __nv_bfloat16*)bias, C::kResidual ? (float*)Y : nullptr, ldy,
      (int)M, (int)N, (int)K);
  return mes_host::from_cuda(cudaGetLastError());
}

// Pair kernel launch: clusters of two CTAs, as many pairs as can be resident at once
// (at most one per two SMs) and no more than there are pair tiles.  PANEL: `w` is the bf16
// weight panel W^T [N, K] (qzeros / scales unused); otherwise the kernel-layout words.
template <int EPI, bool PANEL>
int launch_gemm_pair(const void* X, int64_t ldx, const void* w, const int32_t* qzeros,
                     const void* scales, const void* bias, void* Y, int64_t ldy, int64_t M,
                     int64_t N, int64_t K, cudaStream_t stream) {
  using C = QCfg<EPI, PANEL>;
  auto kern = awq_gemm_pair_kernel<EPI, PANEL>;
  static std::atomic<uint64_t> attr_done{0};
  const int st = mes_host::once_per_device(attr_done, [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) == cudaSuccess
               ? MES_OK : MES_ERR_CUDA;
  });
  if (st != MES_OK) return st;
  CUtensorMap mx, mw, ms, mz, my;
  if (!mes_host::make_map_2d(&mx, X, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, ldx, C::kHalfT,
                             kBK, CU_TENSOR_MAP_SWIZZLE_128B))
    return MES_ERR_INVALID;
  if constexpr (PANEL) {
    if (!mes_host::make_map_2d(&mw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, K, kBN, kBK,
                               CU_TENSOR_MAP_SWIZZLE_128B))
      return MES_ERR_INVALID;
    ms = mw;  // unused by the panel variant
    mz = mw;
  } else {
    if (!mes_host::make_map_2d(&mw, w, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, K / 8, N, N, kBK / 8, kBN,
                               CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !mes_host::make_map_2d(&ms, scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, K / kGroup, N, N, 1,
                               kBN, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !mes_host::make_map_2d(&mz, qzeros, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, K / kGroup, N / 8,
                               N / 8, 1, kBN / 8, CU_TENSOR_MAP_SWIZZLE_NONE))
      return MES_ERR_INVALID;
  }
  if (!make_out_map(&my, mx, EPI, Y, M, N, ldy, C::kChunk)) return MES_ERR_INVALID;
  // The residual epilogue adds into R with TMA reduce-adds when R's rows start on 16-byte
  // boundaries (else it reads and writes R from registers).
  int res_tma = 0;
  if constexpr (C::kResidual) {
    if ((reinterpret_cast<uintptr_t>(Y) & 15) == 0 && ldy % 4 == 0 &&
        mes_host::make_map_2d(&my, Y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, M, N, ldy, C::kChunk, 32,
                              CU_TENSOR_MAP_SWIZZLE_NONE))
      res_tma = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(2, 1, 1);
  // Resident pairs, queried once per device.
  static std::atomic<int> clusters_by_dev[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MES_ERR_CUDA;
  int clusters = clusters_by_dev[dev & 63].load(std::memory_order_relaxed);
  if (clusters <= 0) {
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters < 1)
      return MES_ERR_CUDA;
    clusters_by_dev[dev & 63].store(clusters, std::memory_order_relaxed);
  }
  const int64_t num_n = N / C::kTileN;
  const int64_t tiles = num_n * ((M + C::kTileT - 1) / C::kTileT);
  const int64_t max_pairs = clusters < mes_host::persistent_ctas() / 2 ? clusters : mes_host::persistent_ctas() / 2;
  // A last round of at most half the pairs runs as half tiles on twice as many pairs.
  static const bool half_tail = [] {
    const char* v = getenv("MES_GEMM_HALF_TAIL");
    return !(v && atoi(v) == 0);
  }();
  const int64_t left = tiles % max_pairs;
  const int64_t full = (half_tail && left != 0 && 2 * left <= max_pairs) ? tiles - left : tiles;
  const int64_t items = full + 2 * (tiles - full);
  const int64_t pairs = items < max_pairs ? items : max_pairs;
  // Band of feature tiles walked at a time: the panel rows of a band (about 40 MB at most)
  // stay in L2 while the token tiles pass them.  The packed weights are 4x smaller and are
  // walked in one band.
  int64_t band = num_n;
  if (PANEL) {
    band = (40ll << 20) / ((int64_t)C::kTileN * K * 2);
    band = band < 1 ? 1 : (band > num_n ? num_n : band);
  }
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mx, mw, ms, mz, my, (const __nv_bfloat16*)bias,
                         C::kResidual || C::kSilu ? (float*)Y : nullptr, ldy, (int)M, (int)N, (int)K,
                         (int)band, (int)full, (int)items, res_tma);
  if (e != cudaSuccess) return MES_ERR_CUDA;
  return mes_host::from_cuda(cudaGetLastError());
}

// Weight panels W^T [N_i, K_i] bf16 of up to kMaxPanels GEMMs in one launch (see
// awq_panel_kernel).
int launch_panels(int count, const int32_t* const* qw, const int32_t* const* qzeros,
                  const void* const* scales, const int64_t* K, const int64_t* N,
                  void* const* panels, cudaStream_t stream) {
  if (count < 1 || count > kMaxPanels) return MES_ERR_INVALID;
  PanelJobs jobs = {};
  int64_t blocks = 0;
  for (int i = 0; i < count; ++i) {
    if (!qw[i] || !qzeros[i] || !scales[i] || !panels[i]) return MES_ERR_INVALID;
    if (K[i] <= 0 || N[i] <= 0 || K[i] % kGroup || N[i] % 8 || K[i] > (1 << 24) || N[i] > (1 << 24))
      return MES_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(panels[i]) & 15) || (reinterpret_cast<uintptr_t>(qw[i]) & 3) ||
        (reinterpret_cast<uintptr_t>(qzeros[i]) & 3) || (reinterpret_cast<uintptr_t>(scales[i]) & 1))
      return MES_ERR_ALIGN;
    PanelJob& j = jobs.job[i];
    j.qw = (const uint32_t*)qw[i];
    j.qzeros = qzeros[i];
    j.scales = (const uint16_t*)scales[i];
    j.out = (uint4*)panels[i];
    j.K = (int)K[i];
    j.N = (int)N[i];
    j.kblocks = (int)((K[i] / 8 + 31) / 32);
    j.first_block = (int)blocks;
    blocks += (int64_t)j.kblocks * (N[i] / 8);
  }
  if (blocks > (1ll << 31) - 1) return MES_ERR_INVALID;
  jobs.count = count;
  awq_panel_kernel<<<(unsigned)blocks, 256, 0, stream>>>(jobs);
  return mes_host::from_cuda(cudaGetLastError());
}

int launch_panel(const int32_t* qw, const int32_t* qzeros, const void* scales, int64_t N,
                 int64_t K, void* panel, cudaStream_t stream) {
  return launch_panels(1, &qw, &qzeros, &scales, &K, &N, &panel, stream);
}

// Whether the GEMM of this shape takes the panel path when given a workspace: batches of
// more than 256 tokens (the batches the persistent kernels serve), N a multiple of the pair
// tile, and the panel grid within the launch limits.  MES_GEMM_PANEL=0 (read once) turns
// the path off, for comparisons.
// Batches above this many tokens run on a weight panel (when the caller gives a workspace);
// up to it, the dequantising CTA-pair kernel is faster than building the panel (measured
// per call: 0.71-0.96 of the panel path's time at 512-1024 tokens, even at 2048).
constexpr int64_t kPanelMinTokens = 1024;

bool panel_path(int64_t M, int64_t N, int64_t K) {
  static const bool enabled = [] {
    const char* v = getenv("MES_GEMM_PANEL");
    return !(v && atoi(v) == 0);
  }();
  return enabled && M > kPanelMinTokens && N % (2 * kBN) == 0 && N <= (1 << 24) && K <= (1 << 24);
}

// Tile configuration for M > 64 tokens.  The environment variable MES_GEMM_CONFIG (read
// once) selects among the compiled variants for tuning:
//   0 (default) the residual epilogue on CTA pairs where N is a multiple of 256, the other
//     epilogues on single CTAs (measured at M = 20000: residual N = 1024, K = 2048 865 vs
//     788 TFLOP/s; bf16 N = 6144, K = 1024 1138 vs 1170; SiLU 1117 vs 1159);
//   1 persistent single CTA, 192 tokens, dequantised A in TMEM;
//   2 one 256-token tile per CTA (the default too for M <= 256 while the tiles number at
//     most half the SMs; K is then split over clusters);
//   3 persistent single CTA, 256 tokens, dequantised A in shared memory;
//   4 CTA pairs wherever N is a multiple of 256.
// Narrower single-CTA tiles do not pay: a tile's time is set by its 128 x K weights far
// more than by its token count (measured 1087 / 871 / 622 TFLOP/s for 256 / 192 / 128
// tokens at M = 20000, N = 6144, K = 1024), so the widest tile wins even where a narrower
// one would fill the last wave better.
int large_m_config() {
  static int cfg = [] {
    const char* v = getenv("MES_GEMM_CONFIG");
    int c = v ? atoi(v) : 0;
    return (c < 0 || c > 4) ? 0 : c;
  }();
  return cfg;
}

template <int EPI>
int dispatch_gemm(const void* X, int64_t ldx, const int32_t* qw, const int32_t* qzeros,
                  const void* scales, const void* bias, void* Y, int64_t ldy, int64_t M,
                  int64_t N, int64_t K, void* panel, int64_t panel_bytes, bool ws_aware,
                  cudaStream_t s) {
  if (M <= 16) return launch_gemm<16, 16, 4, EPI, 8>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
  if (M <= 32) return launch_gemm<32, 11, 4, EPI, 8>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
  if (M <= 64) return launch_gemm<64, 7, 4, EPI, 8>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
  const int config = large_m_config();
  // One 256-token tile row that covers at most half the SMs: one tile per CTA with K split
  // over clusters keeps the SMs busy that a persistent kernel would leave idle.  Larger M
  // stays on the persistent kernels, so every batch of more than 256 tokens accumulates
  // each output in the same order (a row's result does not depend on the batch around it).
  if (config == 2 || (config != 1 && M <= 256 && 2 * (N / kBN) <= mes_host::persistent_ctas()))
    return launch_gemm<256, 5, 4, EPI, 8>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
  // Mid-size batches of a workspace-aware caller (mes_awq_gemm_ws), and batches of at most
  // 256 tokens too wide for the one-tile-per-CTA kernel: the dequantising CTA-pair kernel,
  // which runs the same MMAs in the same k order as the panel path above kPanelMinTokens,
  // so a row's result does not depend on which side of it the batch is (measured at 128-256
  // tokens and N = 19456 / 24576 it also beats the single-CTA persistent kernel by 4-6%).
  if (ws_aware && config == 0 && M <= kPanelMinTokens && N % (2 * kBN) == 0)
    return launch_gemm_pair<EPI, false>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
  // Large M with a workspace: dequantise the weights once into a bf16 panel, then run the
  // pair kernel on the panel, so no SM repeats the dequantisation per token tile.
  if (panel && panel_path(M, N, K) && panel_bytes >= N * K * 2) {
    const int st = launch_panel(qw, qzeros, scales, N, K, panel, s);
    if (st != MES_OK) return st;
    return launch_gemm_pair<EPI, true>(X, ldx, panel, qzeros, scales, bias, Y, ldy, M, N, K, s);
  }
  switch (config) {
    case 1: return launch_gemm_persistent<192, 4, 4, EPI, 2>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
    case 3: return launch_gemm_persistent<256, 4, 0, EPI, 2>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
    case 4:
      if (N % (2 * kBN) == 0) return launch_gemm_pair<EPI, false>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
      return launch_gemm_persistent<256, 4, 0, EPI, 2>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
    default:
      if (EPI == kEpiResidual && N % (2 * kBN) == 0)
        return launch_gemm_pair<EPI, false>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
      return launch_gemm_persistent<256, 4, 0, EPI, 2>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
  }
}

// Host checks shared by the GEMM entry points; returns -1 for an empty product (M == 0).
int check_gemm_args(const void* X, int64_t ldx, const int32_t* qw, const int32_t* qzeros,
                    const void* scales, const void* Y, int64_t ldy, int64_t M, int64_t N,
                    int64_t K, int group_size, int y_elem_align, int64_t y_cols) {
  if (M < 0 || N <= 0 || K <= 0 || N % kBN || K % kGroup || group_size != kGroup)
    return MES_ERR_INVALID;
  if (N > (1 << 30) || K > (1 << 30) || M > (1LL << 31) - 256) return MES_ERR_INVALID;
  if (ldx < K || ldy < y_cols || ldx % 8 || ldy % y_elem_align) return MES_ERR_INVALID;
  if (M == 0) return -1;
  if (!X || !qw || !qzeros || !scales || !Y) return MES_ERR_INVALID;
  return MES_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
inline bool aligned_to(const void* p, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0;
}

}  // namespace

extern "C" int mes_gemm_take_error(int* code) {
  int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_err_gemm, sizeof(int));
  if (e != cudaSuccess) return MES_ERR_CUDA;
  e = cudaMemcpyToSymbol(g_err_gemm, &zero, sizeof(int));
  *code = v;
  return mes_host::from_cuda(e);
}

extern "C" int mes_awq_repack(const int32_t* qweight, int64_t K, int64_t N, int32_t* qweight_mes,
                              void* stream) {
  if (K <= 0 || N <= 0 || K % kGroup || N % 8 || !qweight || !qweight_mes) return MES_ERR_INVALID;
  if (!aligned_to(qweight, 4) || !aligned_to(qweight_mes, 4)) return MES_ERR_ALIGN;
  const int64_t total = (K / 8) * N;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 65535) blocks = 65535;
  awq_repack_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      (const uint32_t*)qweight, K, N, (uint32_t*)qweight_mes);
  return mes_host::from_cuda(cudaGetLastError());
}

extern "C" int mes_awq_dequant(const int32_t* qweight_mes, const int32_t* qzeros, const void* scales,
                               int64_t K, int64_t N, int group_size, void* w_out, void* stream) {
  if (K <= 0 || N <= 0 || K % kGroup || N % 8 || group_size != kGroup) return MES_ERR_INVALID;
  if (!qweight_mes || !qzeros || !scales || !w_out) return MES_ERR_INVALID;
  if (!aligned16(w_out) || !aligned_to(qweight_mes, 4) || !aligned_to(qzeros, 4) ||
      !aligned_to(scales, 2))
    return MES_ERR_ALIGN;
  const int64_t total = (K / 8) * N;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 65535) blocks = 65535;
  awq_dequant_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      (const uint32_t*)qweight_mes, qzeros, (const uint16_t*)scales, K, N, (uint4*)w_out);
  return mes_host::from_cuda(cudaGetLastError());
}

extern "C" int64_t mes_awq_gemm_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0 || N % kBN || K % kGroup) return 0;
  return panel_path(M, N, K) ? N * K * 2 : 0;
}

namespace {

// The GEMM entry points.  `ws_aware`: the caller is mes_awq_gemm_ws, which sizes its
// workspace with mes_awq_gemm_workspace_size (the three original entry points keep their
// kernels for every M).
int gemm_entry(int epilogue, const void* X, int64_t ldx, const int32_t* qweight_mes,
               const int32_t* qzeros, const void* scales, const void* bias, void* Y, int64_t ldy,
               int64_t M, int64_t N, int64_t K, int group_size, void* workspace,
               int64_t workspace_bytes, bool ws_aware, void* stream) {
  if (epilogue < kEpiBf16 || epilogue > kEpiSilu || workspace_bytes < 0) return MES_ERR_INVALID;
  if (epilogue == kEpiSilu && bias) return MES_ERR_INVALID;
  const int st = check_gemm_args(X, ldx, qweight_mes, qzeros, scales, Y, ldy, M, N, K, group_size,
                                 epilogue == kEpiResidual ? 1 : 8,
                                 epilogue == kEpiSilu ? N / 2 : N);
  if (st != MES_OK) return st < 0 ? MES_OK : st;
  const bool y_ok = epilogue == kEpiResidual ? (reinterpret_cast<uintptr_t>(Y) & 3) == 0 : aligned16(Y);
  if (!aligned16(X) || !aligned16(qweight_mes) || !aligned16(qzeros) || !aligned16(scales) || !y_ok ||
      !aligned_to(bias, 2))
    return MES_ERR_ALIGN;
  if (workspace && !aligned16(workspace)) return MES_ERR_ALIGN;
  if (!workspace) workspace_bytes = 0;
  cudaStream_t s = (cudaStream_t)stream;
  switch (epilogue) {
    case kEpiBf16:
      return dispatch_gemm<kEpiBf16>(X, ldx, qweight_mes, qzeros, scales, bias, Y, ldy, M, N, K,
                                     workspace, workspace_bytes, ws_aware, s);
    case kEpiResidual:
      return dispatch_gemm<kEpiResidual>(X, ldx, qweight_mes, qzeros, scales, bias, Y, ldy, M, N,
                                         K, workspace, workspace_bytes, ws_aware, s);
    default:
      return dispatch_gemm<kEpiSilu>(X, ldx, qweight_mes, qzeros, scales, nullptr, Y, ldy, M, N, K,
                                     workspace, workspace_bytes, ws_aware, s);
  }
}

}  // namespace

extern "C" int mes_awq_gemm_ws(int epilogue, const void* X, int64_t ldx, const int32_t* qweight_mes,
                               const int32_t* qzeros, const void* scales, const void* bias, void* Y,
                               int64_t ldy, int64_t M, int64_t N, int64_t K, int group_size,
                               void* workspace, int64_t workspace_bytes, void* stream) {
  return gemm_entry(epilogue, X, ldx, qweight_mes, qzeros, scales, bias, Y, ldy, M, N, K,
                    group_size, workspace, workspace_bytes, true, stream);
}

extern "C" int mes_awq_gemm(const void* X, int64_t ldx, const int32_t* qweight_mes,
                            const int32_t* qzeros, const void* scales, const void* bias, void* Y,
                            int64_t ldy, int64_t M, int64_t N, int64_t K, int group_size,
                            void* stream) {
  return gemm_entry(kEpiBf16, X, ldx, qweight_mes, qzeros, scales, bias, Y, ldy, M, N, K,
                    group_size, nullptr, 0, false, stream);
}

extern "C" int mes_awq_gemm_residual(const void* X, int64_t ldx, const int32_t* qweight_mes,
                                     const int32_t* qzeros, const void* scales, const void* bias,
                                     float* R, int64_t ldr, int64_t M, int64_t N, int64_t K,
                                     int group_size, void* stream) {
  return gemm_entry(kEpiResidual, X, ldx, qweight_mes, qzeros, scales, bias, R, ldr, M, N, K,
                    group_size, nullptr, 0, false, stream);
}

extern "C" int mes_awq_gemm_silu(const void* X, int64_t ldx, const int32_t* qweight_mes,
                                 const int32_t* qzeros, const void* scales, void* Y, int64_t ldy,
                                 int64_t M, int64_t N, int64_t K, int group_size, void* stream) {
  return gemm_entry(kEpiSilu, X, ldx, qweight_mes, qzeros, scales, nullptr, Y, ldy, M, N, K,
                    group_size, nullptr, 0, false, stream);
}

extern "C" int mes_awq_panels(int count, const int32_t* const* qweight_mes,
                              const int32_t* const* qzeros, const void* const* scales,
                              const int64_t* K, const int64_t* N, void* const* panels,
                              void* stream) {
  if (!qweight_mes || !qzeros || !scales || !K || !N || !panels) return MES_ERR_INVALID;
  return launch_panels(count, qweight_mes, qzeros, scales, K, N, panels, (cudaStream_t)stream);
}

extern "C" int mes_awq_gemm_on_panel(int epilogue, const void* X, int64_t ldx, const void* panel,
                                     const void* bias, void* Y, int64_t ldy, int64_t M, int64_t N,
                                     int64_t K, void* stream) {
  if (epilogue < kEpiBf16 || epilogue > kEpiSilu) return MES_ERR_INVALID;
  if (epilogue == kEpiSilu && bias) return MES_ERR_INVALID;
  if (M < 0 || N <= 0 || K <= 0 || K % kGroup || ldx < K || ldx % 8) return MES_ERR_INVALID;
  const int64_t y_cols = epilogue == kEpiSilu ? N / 2 : N;
  if (ldy < y_cols || (epilogue != kEpiResidual && ldy % 8)) return MES_ERR_INVALID;
  if (M == 0) return MES_OK;
  if (!panel_path(M, N, K) || !X || !panel || !Y) return MES_ERR_INVALID;
  const bool y_ok = epilogue == kEpiResidual ? (reinterpret_cast<uintptr_t>(Y) & 3) == 0 : aligned16(Y);
  if (!aligned16(X) || !aligned16(panel) || !y_ok || !aligned_to(bias, 2)) return MES_ERR_ALIGN;
  cudaStream_t s = (cudaStream_t)stream;
  switch (epilogue) {
    case kEpiBf16:
      return launch_gemm_pair<kEpiBf16, true>(X, ldx, panel, nullptr, nullptr, bias, Y, ldy, M, N, K, s);
    case kEpiResidual:
      return launch_gemm_pair<kEpiResidual, true>(X, ldx, panel, nullptr, nullptr, bias, Y, ldy, M, N, K, s);
    default:
      return launch_gemm_pair<kEpiSilu, true>(X, ldx, panel, nullptr, nullptr, nullptr, Y, ldy, M, N, K, s);
  }
}
