// Varlen causal GQA prefill attention on tcgen05 / TMEM (head_dim 128).
//
// Persistent kernel, one CTA per SM.  Work items are (sequence, 128-row query tile, query
// head), produced on the device by mes_varlen_schedule in order of decreasing causal
// cost; CTA b takes items b, b + grid, ...  Per item:
//   * warp 0 (TMA) loads the Q tile (128 x 128 bf16, two 64-column boxes, 128-byte swizzle)
//     and, for each key tile i = 0 .. qtile, the K and V tiles into a 2-stage ring;
//   * warp 1 (one thread) issues S_i = Q K_i^T into one of two TMEM S buffers
//     (M = N = 128, K = 16 x 8), and O += P_{i-1} V_{i-1} with P read from TMEM and V from
//     smem in MN-major form;
//   * warps 2..5 (one query row per thread) run the online softmax in the exp2 domain:
//     tcgen05.ld of S, causal mask on the diagonal tile, running max / sum, P = exp2(...)
//     written back to TMEM as bf16 (tcgen05.st), and rescale O in TMEM only when the
//     running max grew by more than 2^8; finally O / l is stored as bf16.
// Scores of rows past the end of the sequence are computed but never stored; keys past
// the end are excluded by the causal mask of the diagonal tile.
#include "common.cuh"

namespace {

__device__ int g_err_attn = 0;

constexpr int kD = 128;
constexpr int kTile = 128;
constexpr int kKVStages = 2;
constexpr int kThreads = 192;

constexpr int kQBytes = kTile * kD * 2;   // 32 KB (two 16 KB boxes)
constexpr int kKVBytes = kTile * kD * 2;  // 32 KB each for K and V
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kQBytes;
constexpr int kOffV = kOffK + kKVStages * kKVBytes;
constexpr int kOffBar = kOffV + kKVStages * kKVBytes;
constexpr int kSmem = kOffBar + 256 + 1024;

// TMEM columns: S0 [0,128), S1 [128,256), O [256,384), P [384,448).
constexpr uint32_t kColS = 0, kColO = 256, kColP = 384;
constexpr uint32_t kTmemCols = 512;

__global__ void __launch_bounds__(kThreads, 1)
varlen_attention_kernel(const __grid_constant__ CUtensorMap map_qkv, __nv_bfloat16* __restrict__ out,
                        const int* __restrict__ hdr, const int* __restrict__ cu,
                        const int2* __restrict__ items, int Hq, int Hkv, float scale_log2) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem + kOffQ;
  uint8_t* ks = smem + kOffK;
  uint8_t* vs = smem + kOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;               // [kKVStages]
  uint64_t* v_full = bars + 2 + kKVStages;   // [kKVStages]
  uint64_t* kv_empty = bars + 2 + 2 * kKVStages;  // [kKVStages]
  uint64_t* s_full = bars + 2 + 3 * kKVStages;    // [2]
  uint64_t* s_free = s_full + 2;                  // [2]
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 1;
  uint64_t* drain = pv_done + 1;                  // abort path: issued MMAs completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = mes::warp_id(), lane = mes::lane_id();
  const int num_work = hdr[1] * Hq;
  const int rep = Hq / Hkv;

  if (threadIdx.x == 0) {
    mes::mbar_init(q_full, 1);
    mes::mbar_init(q_empty, 1);
    for (int s = 0; s < kKVStages; ++s) {
      mes::mbar_init(&k_full[s], 1);
      mes::mbar_init(&v_full[s], 1);
      mes::mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mes::mbar_init(&s_full[b], 1);
      mes::mbar_init(&s_free[b], 4);
    }
    mes::mbar_init(p_full, 4);
    mes::mbar_init(pv_done, 1);
    mes::mbar_init(drain, 1);
    *abort_flag = 0;
    mes::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) mes::tma_prefetch_desc(&map_qkv);
  if (warp == 1) {
    __syncwarp();
    mes::tmem_alloc(tmem_slot, kTmemCols);
    mes::tmem_relinquish();
  }
  mes::tc_fence_before();
  __syncthreads();
  mes::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------ TMA ----------------------------------------
    if (lane == 0) {
      int n_item = 0, kvit = 0, q_issued = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < num_work && ok; w += gridDim.x, ++n_item) {
        const int2 it = items[w / Hq];
        const int h = w % Hq, g = h / rep;
        const int start = cu[it.x];
        const int q0 = start + it.y * kTile;
        if (n_item > 0 && !mes::mbar_wait(q_empty, (n_item - 1) & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) {
          ok = false;
          break;
        }
        ++q_issued;
        mes::mbar_arrive_expect_tx(q_full, kQBytes);
        mes::tma_load_2d(qs, &map_qkv, q_full, h * kD, q0);
        mes::tma_load_2d(qs + kQBytes / 2, &map_qkv, q_full, h * kD + 64, q0);
        const int kcol = (Hq + g) * kD, vcol = (Hq + Hkv + g) * kD;
        for (int i = 0; i <= it.y; ++i, ++kvit) {
          const int st = kvit % kKVStages;
          if (kvit >= kKVStages &&
              !mes::mbar_wait(&kv_empty[st], ((kvit / kKVStages) & 1) ^ 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          const int k0 = start + i * kTile;
          uint8_t* kd = ks + st * kKVBytes;
          uint8_t* vd = vs + st * kKVBytes;
          mes::mbar_arrive_expect_tx(&k_full[st], kKVBytes);
          mes::tma_load_2d(kd, &map_qkv, &k_full[st], kcol, k0);
          mes::tma_load_2d(kd + kKVBytes / 2, &map_qkv, &k_full[st], kcol + 64, k0);
          mes::mbar_arrive_expect_tx(&v_full[st], kKVBytes);
          mes::tma_load_2d(vd, &map_qkv, &v_full[st], vcol, k0);
          mes::tma_load_2d(vd + kKVBytes / 2, &map_qkv, &v_full[st], vcol + 64, k0);
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA exits: the last Q tile and the
        // last kKVStages K and V tiles (bounded, one deadline for all).
        const uint64_t t0 = mes::globaltimer_ns();
        auto landed = [&](uint64_t* bar, int n, int stages) {
          while (!mes::mbar_try_wait(&bar[n % stages], (n / stages) & 1) &&
                 mes::globaltimer_ns() - t0 < mes::kWaitLimitNs) {
          }
        };
        if (q_issued > 0) landed(q_full, q_issued - 1, 1);
        for (int i = kvit - kKVStages < 0 ? 0 : kvit - kKVStages; i < kvit; ++i) {
          landed(k_full, i, kKVStages);
          landed(v_full, i, kKVStages);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------ MMA ----------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = mes::idesc_bf16_f32(kTile, kTile, false);
      constexpr uint32_t idesc_o = mes::idesc_bf16_f32(kTile, kD, true);
      const uint32_t q_addr = mes::smem_u32(qs), k_addr = mes::smem_u32(ks), v_addr = mes::smem_u32(vs);
      int n_item = 0, it = 0;  // `it`: key tiles processed by this CTA so far
      bool ok = true;
      for (int w = blockIdx.x; w < num_work && ok; w += gridDim.x, ++n_item) {
        const int nt = items[w / Hq].y + 1;
        if (!mes::mbar_wait(q_full, n_item & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
        for (int i = 0; i <= nt && ok; ++i) {
          if (i < nt) {
            // S_i = Q K_i^T
            const int t = it + i, sb = t & 1, st = t % kKVStages;
            if (t >= 2 && !mes::mbar_wait(&s_free[sb], ((t >> 1) - 1) & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
            if (!mes::mbar_wait(&k_full[st], (t / kKVStages) & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
            mes::tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              const uint32_t off = (kk >> 2) * (kQBytes / 2) + (kk & 3) * 32;
              mes::mma_ss(tmem + kColS + sb * 128, mes::smem_desc_sw128(q_addr + off, 16, 1024),
                          mes::smem_desc_sw128(k_addr + st * kKVBytes + off, 16, 1024), idesc_s, kk != 0);
            }
            mes::tc_commit(&s_full[sb]);
            if (i == nt - 1) mes::tc_commit(q_empty);
          }
          if (i > 0) {
            // O += P_{i-1} V_{i-1}
            const int t = it + i - 1, st = t % kKVStages;
            if (!mes::mbar_wait(p_full, t & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
            if (!mes::mbar_wait(&v_full[st], (t / kKVStages) & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
            mes::tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < kTile / 16; ++kk) {
              // V tile: rows = keys (the MMA's K), 128-byte rows of 64 head-dim elements; the
              // second 64-column box is the next MN block (LBO = 16 KB), 8-row atoms along K
              // are 1 KB apart (SBO).
              const uint64_t vdesc =
                  mes::smem_desc_sw128(v_addr + st * kKVBytes + kk * 16 * 128, kKVBytes / 2, 1024);
              mes::mma_ts(tmem + kColO, tmem + kColP + kk * 8, vdesc, idesc_o, (i - 1 > 0 || kk > 0));
            }
            mes::tc_commit(pv_done);
            mes::tc_commit(&kv_empty[st]);
          }
        }
        it += nt;
      }
      if (!ok) {
        // Wait (bounded) until every MMA issued so far has completed.
        mes::tc_commit(drain);
        const uint64_t t0 = mes::globaltimer_ns();
        while (!mes::mbar_try_wait(drain, 0) && mes::globaltimer_ns() - t0 < mes::kWaitLimitNs) {
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------- softmax -------------------------------------
    const int q = warp & 3;
    const int r = q * 32 + lane;  // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    int n_item = 0, it = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < num_work && ok; w += gridDim.x, ++n_item) {
      const int2 item = items[w / Hq];
      const int h = w % Hq;
      const int start = cu[item.x], len = cu[item.x + 1] - start;
      const int nt = item.y + 1;
      float m = -INFINITY, l = 0.f;
      for (int i = 0; i < nt; ++i) {
        const int t = it + i, sb = t & 1;
        if (!mes::mbar_wait_warp(&s_full[sb], (t >> 1) & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
        mes::tc_fence_after();
        float s[kTile];
#pragma unroll
        for (int c = 0; c < kTile; c += 32) {
          uint32_t v[32];
          mes::tmem_ld32(tmem + lane_off + kColS + sb * 128 + c, v);
          mes::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) s[c + j] = __uint_as_float(v[j]);
        }
        mes::tc_fence_before();
        __syncwarp();
        if (lane == 0) mes::mbar_arrive(&s_free[sb]);
        __syncwarp();
        // Causal mask on the diagonal tile: key c is visible to row r iff c <= r.
        if (i == nt - 1) {
#pragma unroll
          for (int c = 0; c < kTile; ++c)
            if (c > r) s[c] = -INFINITY;
        }
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < kTile; ++c) mx = fmaxf(mx, s[c]);
        mx *= scale_log2;
        // PV_{i-1} must be done before O is rescaled or P overwritten.
        if (i > 0 && !mes::mbar_wait_warp(pv_done, (t - 1) & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
        mes::tc_fence_after();
        if (i == 0) {
          m = mx;
        } else if (__any_sync(0xffffffffu, mx > m + 8.0f)) {
          // Warp-uniform decision (tcgen05.ld/st are warp-collective): every row of the
          // warp moves to max(m, mx); rows whose maximum did not grow scale by 1.
          const float mn = fmaxf(m, mx);
          const float f = exp2f(m - mn);
          l *= f;
          m = mn;
#pragma unroll 1
          for (int c = 0; c < kD; c += 32) {
            uint32_t v[32];
            mes::tmem_ld32(tmem + lane_off + kColO + c, v);
            mes::tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * f);
            mes::tmem_st32(tmem + lane_off + kColO + c, v);
          }
        }
        float sum = 0.f;
        uint32_t plo[32], phi[32];
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          const float p0 = exp2f(fmaf(s[c], scale_log2, -m));
          const float p1 = exp2f(fmaf(s[c + 1], scale_log2, -m));
          sum += p0 + p1;
          plo[c / 2] = mes::pack_bf16x2(p0, p1);
        }
#pragma unroll
        for (int c = 64; c < kTile; c += 2) {
          const float p0 = exp2f(fmaf(s[c], scale_log2, -m));
          const float p1 = exp2f(fmaf(s[c + 1], scale_log2, -m));
          sum += p0 + p1;
          phi[(c - 64) / 2] = mes::pack_bf16x2(p0, p1);
        }
        l += sum;
        mes::tmem_st32(tmem + lane_off + kColP, plo);
        mes::tmem_st32(tmem + lane_off + kColP + 32, phi);
        mes::tmem_wait_st();
        mes::tc_fence_before();
        __syncwarp();
        if (lane == 0) mes::mbar_arrive(p_full);
        __syncwarp();
      }
      if (!ok) break;
      // Epilogue: O / l for this item's rows.
      const int tl = it + nt - 1;
      if (!mes::mbar_wait_warp(pv_done, tl & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
      mes::tc_fence_after();
      const int row_in_seq = item.y * kTile + r;
      const bool valid = row_in_seq < len;
      const float inv = 1.0f / l;
      uint4* dst = reinterpret_cast<uint4*>(out + ((int64_t)(start + row_in_seq) * Hq + h) * kD);
#pragma unroll 1
      for (int c = 0; c < kD; c += 32) {
        uint32_t v[32];
        mes::tmem_ld32(tmem + lane_off + kColO + c, v);
        mes::tmem_wait_ld();
        if (valid) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 o;
            o.x = mes::pack_bf16x2(__uint_as_float(v[j + 0]) * inv, __uint_as_float(v[j + 1]) * inv);
            o.y = mes::pack_bf16x2(__uint_as_float(v[j + 2]) * inv, __uint_as_float(v[j + 3]) * inv);
            o.z = mes::pack_bf16x2(__uint_as_float(v[j + 4]) * inv, __uint_as_float(v[j + 5]) * inv);
            o.w = mes::pack_bf16x2(__uint_as_float(v[j + 6]) * inv, __uint_as_float(v[j + 7]) * inv);
            dst[(c + j) / 8] = o;
          }
        }
      }
      mes::tc_fence_before();
      it += nt;
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

// =========================================================================================
// Head-pair kernel (query heads per KV head even): two query heads of one KV group share
// every K/V tile.  Per item (sequence, 128-row query tile, head pair):
//   * warp 8 (TMA) loads both Q tiles (64 KB) and, for key tiles 0 .. qtile, K and V into
//     separate 2-stage rings;
//   * warp 9 (one thread) issues, in this order,
//       S0_0, S1_0, { PV0_j, S0_{j+1}, PV1_j, S1_{j+1} } for j = 0 .. qtile,
//     so the tensor core runs tile 1's MMAs while warpgroup 0 runs the softmax of tile 0
//     and the other way round;
//   * warps 0-3 / 4-7 run the online softmax of head 0 / head 1 of the pair (one query row
//     per thread), write P (bf16) over the first 64 columns of their own S buffer, rescale
//     O in TMEM when the running maximum grew by more than 2^8, and store O / l at the end.
// TMEM: S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512); P_b aliases S_b.
// tcgen05.mma operations issued by one thread execute in issue order, so S_b(j+1), issued
// after PV_b(j), overwrites P_b(j) only after PV_b(j) has read it, and the commit that
// signals S_b(j+1) also covers PV_b(j): when warpgroup b sees S_b(j+1), O_b holds every
// P_b(i) V_i for i <= j and no MMA writes O_b until warpgroup b publishes P_b(j+1).
//
// exp2 runs on two units: the special-function unit (ex2.approx) and, for kPolyPairs of
// every 8 element pairs, the FMA pipe with 2^x = 2^n * q(x - n), n = round(x), and q a
// degree-3 polynomial for 2^f on [-1/2, 1/2] fitted for minimum maximum relative error
// (Lawson's iteratively reweighted least squares; max relative error 7.5e-5, against the
// 2^-9 relative rounding of P to bf16).  Packed f32x2 FMA / add halve the issue count of
// the element-wise work.
constexpr int kPThreads = 384;  // warps 0-7 softmax, 8 TMA, 9 MMA, 10-11 idle
// Register split (setmaxnreg acts on whole warpgroups): softmax warpgroups grow to
// kSoftmaxRegs, warpgroup 2 shrinks to kOtherRegs.  The host launches the kernel only when
// the registers it was compiled for cover the split (otherwise setmaxnreg.inc would wait).
constexpr int kSoftmaxRegs = 200;
constexpr int kOtherRegs = 104;
constexpr int kPOffQ = 0;                                   // Q0 | Q1, 2 x 32 KB
constexpr int kPOffK = kPOffQ + 2 * kQBytes;
constexpr int kPOffV = kPOffK + kKVStages * kKVBytes;
constexpr int kPOffBar = kPOffV + kKVStages * kKVBytes;
// O staging for the TMA store of the epilogue: 4 KB per softmax warp (32 rows x 64 columns
// bf16, 128-byte swizzle), 1024-byte aligned.
constexpr int kPOffStage = kPOffBar + 1024;
constexpr int kStageBytes = 32 * 64 * 2;
constexpr int kPSmem = kPOffStage + 8 * kStageBytes + 1024;
static_assert(kPSmem <= 232448, "shared memory");

__device__ __forceinline__ uint64_t f2_bits(float2 v) {
  return (uint64_t)__float_as_uint(v.x) | ((uint64_t)__float_as_uint(v.y) << 32);
}
__device__ __forceinline__ float2 bits_f2(uint64_t b) {
  return make_float2(__uint_as_float((uint32_t)b), __uint_as_float((uint32_t)(b >> 32)));
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return bits_f2(d);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float ex2_sfu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x for a pair on the FMA pipe (x <= 2^22); inputs below -126 give about 2^-126.
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: adding it rounds to an integer
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 t = fadd2(x, make_float2(kRound, kRound));
  const float2 n = fadd2(t, make_float2(-kRound, -kRound));
  const float2 f = fadd2(x, make_float2(-n.x, -n.y));
  float2 q = ffma2(make_float2(0x1.c3f76p-5f, 0x1.c3f76p-5f), f, make_float2(0x1.f0de1cp-3f, 0x1.f0de1cp-3f));
  q = ffma2(q, f, make_float2(0x1.62f31ap-1f, 0x1.62f31ap-1f));
  q = ffma2(q, f, make_float2(0x1.fff692p-1f, 0x1.fff692p-1f));
  // The low bits of t hold n; shifting them into the exponent field scales q by 2^n.
  return make_float2(__uint_as_float(__float_as_uint(q.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(t.y) << 23)));
}

// Work index of the k-th item of CTA b: rows of the descending-cost list are dealt out
// left to right, then right to left, so every CTA's total cost stays close to the mean.
__device__ __forceinline__ int snake(int k, int b, int G) {
  return k * G + ((k & 1) ? (G - 1 - b) : b);
}

template <int kPolyPairs>
__global__ void __launch_bounds__(kPThreads, 1)
varlen_attention_pair_kernel(const __grid_constant__ CUtensorMap map_qkv,
                             const __grid_constant__ CUtensorMap map_out,
                             __nv_bfloat16* __restrict__ out, const int* __restrict__ hdr,
                             const int* __restrict__ cu, const int2* __restrict__ items, int Hq,
                             int Hkv, float scale_log2, int l2_hints) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem + kPOffQ;
  uint8_t* ks = smem + kPOffK;
  uint8_t* vs = smem + kPOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;    // [kKVStages]
  uint64_t* k_empty = bars + 4;   // [kKVStages]
  uint64_t* v_full = bars + 6;    // [kKVStages]
  uint64_t* v_empty = bars + 8;   // [kKVStages]
  uint64_t* s_full = bars + 10;   // [2] per head of the pair
  uint64_t* p_full = bars + 12;   // [2]
  uint64_t* o_full = bars + 14;   // [2]
  uint64_t* drain = bars + 16;    // abort path: issued MMAs completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* turn = bars + 18;     // [2] softmax warpgroup b may run its exp2 phase

  const int warp = mes::warp_id(), lane = mes::lane_id();
  const int npairs = Hq / 2;
  const int num_work = hdr[1] * npairs;
  const int rep = Hq / Hkv;

  if (threadIdx.x == 0) {
    mes::mbar_init(q_full, 1);
    mes::mbar_init(q_empty, 1);
    for (int s = 0; s < kKVStages; ++s) {
      mes::mbar_init(&k_full[s], 1);
      mes::mbar_init(&k_empty[s], 1);
      mes::mbar_init(&v_full[s], 1);
      mes::mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mes::mbar_init(&s_full[b], 1);
      mes::mbar_init(&p_full[b], 4);
      mes::mbar_init(&o_full[b], 1);
      mes::mbar_init(&turn[b], 4);
    }
    mes::mbar_init(drain, 1);
    *abort_flag = 0;
    mes::fence_barrier_init();
  }
  if (warp == 8 && lane == 0) {
    mes::tma_prefetch_desc(&map_qkv);
    mes::tma_prefetch_desc(&map_out);
  }
  if (warp == 9) {
    __syncwarp();
    mes::tmem_alloc(tmem_slot, kTmemCols);
    mes::tmem_relinquish();
  }
  mes::tc_fence_before();
  __syncthreads();
  mes::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kOtherRegs));
   if (warp == 8) {
    // ------------------------------------ TMA ----------------------------------------
    if (lane == 0) {
      // Each K/V tile is read by every query tile of its sequence, spread over time; each Q
      // tile once.  Keep K/V in L2 in preference to Q.
      const uint64_t pol_kv = mes::l2_policy_evict_last();
      const uint64_t pol_q = mes::l2_policy_evict_first();
      auto load = [&](void* dst, uint64_t* bar, int x, int y, uint64_t pol) {
        if (l2_hints) mes::tma_load_2d_hint(dst, &map_qkv, bar, x, y, pol);
        else mes::tma_load_2d(dst, &map_qkv, bar, x, y);
      };
      int n_item = 0, kt = 0, vt = 0, q_issued = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < num_work && ok; w = snake(++n_item, blockIdx.x, gridDim.x)) {
        const int2 it = items[w / npairs];
        const int h0 = 2 * (w % npairs), g = h0 / rep;
        const int start = cu[it.x];
        const int q0 = start + it.y * kTile;
        if (n_item > 0 && !mes::mbar_wait(q_empty, (n_item - 1) & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) {
          ok = false;
          break;
        }
        ++q_issued;
        mes::mbar_arrive_expect_tx(q_full, 2 * kQBytes);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          load(qs + c * (kQBytes / 2), q_full, h0 * kD + c * 64, q0, pol_q);
        const int kcol = (Hq + g) * kD, vcol = (Hq + Hkv + g) * kD;
        for (int j = 0; j <= it.y; ++j) {
          const int k0 = start + j * kTile;
          const int ks_ = kt % kKVStages, vs_ = vt % kKVStages;
          if (kt >= kKVStages &&
              !mes::mbar_wait(&k_empty[ks_], ((kt / kKVStages) & 1) ^ 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          uint8_t* kd = ks + ks_ * kKVBytes;
          mes::mbar_arrive_expect_tx(&k_full[ks_], kKVBytes);
          load(kd, &k_full[ks_], kcol, k0, pol_kv);
          load(kd + kKVBytes / 2, &k_full[ks_], kcol + 64, k0, pol_kv);
          ++kt;
          if (vt >= kKVStages &&
              !mes::mbar_wait(&v_empty[vs_], ((vt / kKVStages) & 1) ^ 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          uint8_t* vd = vs + vs_ * kKVBytes;
          mes::mbar_arrive_expect_tx(&v_full[vs_], kKVBytes);
          load(vd, &v_full[vs_], vcol, k0, pol_kv);
          load(vd + kKVBytes / 2, &v_full[vs_], vcol + 64, k0, pol_kv);
          ++vt;
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA exits: the last Q tiles and
        // the last kKVStages K and V tiles (bounded, one deadline for all).
        const uint64_t t0 = mes::globaltimer_ns();
        auto landed = [&](uint64_t* bar, int n, int stages) {
          while (!mes::mbar_try_wait(&bar[n % stages], (n / stages) & 1) &&
                 mes::globaltimer_ns() - t0 < mes::kWaitLimitNs) {
          }
        };
        if (q_issued > 0) landed(q_full, q_issued - 1, 1);
        for (int i = kt - kKVStages < 0 ? 0 : kt - kKVStages; i < kt; ++i) landed(k_full, i, kKVStages);
        for (int i = vt - kKVStages < 0 ? 0 : vt - kKVStages; i < vt; ++i) landed(v_full, i, kKVStages);
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------ MMA ----------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = mes::idesc_bf16_f32(kTile, kTile, false);
      constexpr uint32_t idesc_o = mes::idesc_bf16_f32(kTile, kD, true);
      // Descriptors differ only in the start-address field (bits [0,14), address >> 4), and
      // every operand lies below 256 KB, so offsets are added to a base descriptor.
      const uint64_t dq = mes::smem_desc_sw128(mes::smem_u32(qs), 16, 1024);
      const uint64_t dk = mes::smem_desc_sw128(mes::smem_u32(ks), 16, 1024);
      const uint64_t dv = mes::smem_desc_sw128(mes::smem_u32(vs), kKVBytes / 2, 1024);
      auto issue_s = [&](int b, int st) {
        const uint64_t da = dq + (uint32_t)(b * (kQBytes >> 4));
        const uint64_t db = dk + (uint32_t)(st * (kKVBytes >> 4));
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * (kQBytes / 2) + (kk & 3) * 32) >> 4;
          mes::mma_ss(tmem + b * 128, da + off, db + off, idesc_s, kk != 0);
        }
      };
      auto issue_pv = [&](int b, int st, bool acc) {
        // V tile: keys are the MMA's K; 128-byte rows of 64 head-dim elements, the second
        // 64-column box is the next MN block (LBO = 16 KB), 8-row atoms 1 KB apart (SBO).
        const uint64_t dvs = dv + (uint32_t)(st * (kKVBytes >> 4));
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          mes::mma_ts(tmem + 256 + b * 128, tmem + b * 128 + kk * 8, dvs + (uint32_t)(kk * 128),
                      idesc_o, acc || kk > 0);
      };
      int n_item = 0, kt = 0, vt = 0, pt = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < num_work && ok; w = snake(++n_item, blockIdx.x, gridDim.x)) {
        const int nt = items[w / npairs].y + 1;
        if (!mes::mbar_wait(q_full, n_item & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
        if (!mes::mbar_wait(&k_full[kt % kKVStages], (kt / kKVStages) & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
        mes::tc_fence_after();
        issue_s(0, kt % kKVStages);
        mes::tc_commit(&s_full[0]);
        issue_s(1, kt % kKVStages);
        mes::tc_commit(&s_full[1]);
        mes::tc_commit(&k_empty[kt % kKVStages]);
        ++kt;
        if (nt == 1) mes::tc_commit(q_empty);
        for (int j = 0; j < nt; ++j, ++vt, ++pt) {
          const int vst = vt % kKVStages;
          if (!mes::mbar_wait(&p_full[0], pt & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
          if (!mes::mbar_wait(&v_full[vst], (vt / kKVStages) & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
          mes::tc_fence_after();
          issue_pv(0, vst, j > 0);
          if (j == nt - 1) mes::tc_commit(&o_full[0]);
          const bool more = j + 1 < nt;
          if (more) {
            if (!mes::mbar_wait(&k_full[kt % kKVStages], (kt / kKVStages) & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
            mes::tc_fence_after();
            issue_s(0, kt % kKVStages);
            mes::tc_commit(&s_full[0]);
          }
          if (!mes::mbar_wait(&p_full[1], pt & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
          mes::tc_fence_after();
          issue_pv(1, vst, j > 0);
          mes::tc_commit(&v_empty[vst]);
          if (j == nt - 1) mes::tc_commit(&o_full[1]);
          if (more) {
            issue_s(1, kt % kKVStages);
            mes::tc_commit(&s_full[1]);
            mes::tc_commit(&k_empty[kt % kKVStages]);
            ++kt;
            if (j + 1 == nt - 1) mes::tc_commit(q_empty);
          }
        }
      }
      if (!ok) {
        // Wait (bounded) until every MMA issued so far has completed.
        mes::tc_commit(drain);
        const uint64_t t0 = mes::globaltimer_ns();
        while (!mes::mbar_try_wait(drain, 0) && mes::globaltimer_ns() - t0 < mes::kWaitLimitNs) {
        }
      }
    }
    __syncwarp();
   }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // ---------------------------------- softmax -------------------------------------
    const int b = warp >> 2;           // head of the pair
    const int r = (warp & 3) * 32 + lane;  // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + lane_off + b * 128;
    const uint32_t t_o = tmem + lane_off + 256 + b * 128;
    const float2 sc2 = make_float2(scale_log2, scale_log2);
    int n_item = 0, pt = 0;
    bool ok = true;
    bool o_stored = false;  // this warp has TMA stores of O in flight
    for (int w = blockIdx.x; w < num_work && ok; w = snake(++n_item, blockIdx.x, gridDim.x)) {
      const int2 item = items[w / npairs];
      const int h = 2 * (w % npairs) + b;
      const int start = cu[item.x], len = cu[item.x + 1] - start;
      const int nt = item.y + 1;
      float m = 0.f, l = 0.f;
      for (int j = 0; j < nt; ++j, ++pt) {
        if (!mes::mbar_wait_warp(&s_full[b], pt & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
        mes::tc_fence_after();
        float s[kTile];
        {
          uint32_t v0[32], v1[32], v2[32], v3[32];
          mes::tmem_ld32(t_s + 0, v0);
          mes::tmem_ld32(t_s + 32, v1);
          mes::tmem_ld32(t_s + 64, v2);
          mes::tmem_ld32(t_s + 96, v3);
          mes::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            s[c] = __uint_as_float(v0[c]);
            s[32 + c] = __uint_as_float(v1[c]);
            s[64 + c] = __uint_as_float(v2[c]);
            s[96 + c] = __uint_as_float(v3[c]);
          }
        }
        // Causal mask on the diagonal tile: key c is visible to row r iff c <= r.
        if (j == nt - 1) {
#pragma unroll
          for (int c = 0; c < kTile; ++c)
            if (c > r) s[c] = -INFINITY;
        }
        float mq[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) mq[u] = fmaxf(s[2 * u], s[2 * u + 1]);
#pragma unroll
        for (int c = 8; c < kTile; c += 8)
#pragma unroll
          for (int u = 0; u < 4; ++u) mq[u] = fmax3(mq[u], s[c + 2 * u], s[c + 2 * u + 1]);
        float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * scale_log2;
        // Lazy rescale: move to the new maximum only when it grew by more than 2^8 (the
        // decision is warp-uniform because tcgen05.ld/st are warp-collective; rows whose
        // maximum did not grow scale by 1).  O_b is rescaled after P_b is written, when
        // the S registers are dead; no MMA touches O_b before P_b is published.
        float f = 1.0f;
        bool rescale = false;
        if (j == 0) {
          m = mx;
        } else if (__any_sync(0xffffffffu, mx > m + 8.0f)) {
          const float mn = fmaxf(m, mx);
          f = ex2_sfu(m - mn);
          l *= f;
          m = mn;
          rescale = true;
        }
        // The exp2 phases of the two warpgroups take turns (head 0 of step pt, head 1 of
        // step pt, head 0 of step pt + 1, ...): both would otherwise contend for the SM's
        // exp2 unit, finish together and leave the tensor core to run both heads' MMAs while
        // neither softmax can proceed.  Taking turns, one head's exp2 phase runs while the
        // tensor core computes the other head's PV and next S.
        if (b == 1 || pt > 0) {
          const uint32_t par = b == 0 ? ((pt - 1) & 1) : (pt & 1);
          if (!mes::mbar_wait_warp(&turn[b], par, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
        }
        const float2 nm2 = make_float2(-m, -m);
        float2 sum2[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) sum2[u] = make_float2(0.f, 0.f);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = q4 * 32 + 2 * i;
            const float2 x = ffma2(make_float2(s[c], s[c + 1]), sc2, nm2);
            float2 p;
            if ((i & 7) < kPolyPairs) {
              p = ex2_poly2(x);
            } else {
              p.x = ex2_sfu(x.x);
              p.y = ex2_sfu(x.y);
            }
            sum2[i & 3] = fadd2(sum2[i & 3], p);
            pk[i] = mes::pack_bf16x2(p.x, p.y);
          }
          mes::tmem_st16(t_s + q4 * 16, pk);
        }
        __syncwarp();
        if (lane == 0) mes::mbar_arrive(&turn[b ^ 1]);
        const float2 s01 = fadd2(sum2[0], sum2[1]), s23 = fadd2(sum2[2], sum2[3]);
        l += (s01.x + s23.x) + (s01.y + s23.y);
        if (rescale) {
#pragma unroll 1
          for (int c = 0; c < kD; c += 32) {
            uint32_t v[32];
            mes::tmem_ld32(t_o + c, v);
            mes::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * f);
            mes::tmem_st32(t_o + c, v);
          }
        }
        mes::tmem_wait_st();
        mes::tc_fence_before();
        __syncwarp();
        if (lane == 0) mes::mbar_arrive(&p_full[b]);
        __syncwarp();
      }
      if (!ok) break;
      // Epilogue: O / l for this item's rows.
      if (!mes::mbar_wait_warp(&o_full[b], n_item & 1, abort_flag, &g_err_attn, MES_ERR_TIMEOUT)) { ok = false; break; }
      mes::tc_fence_after();
      const int row_in_seq = item.y * kTile + r;
      const bool valid = row_in_seq < len;
      const float inv = 1.0f / l;
      auto scale8 = [&](const uint32_t (&v)[32], int i) {
        uint4 o;
        o.x = mes::pack_bf16x2(__uint_as_float(v[i + 0]) * inv, __uint_as_float(v[i + 1]) * inv);
        o.y = mes::pack_bf16x2(__uint_as_float(v[i + 2]) * inv, __uint_as_float(v[i + 3]) * inv);
        o.z = mes::pack_bf16x2(__uint_as_float(v[i + 4]) * inv, __uint_as_float(v[i + 5]) * inv);
        o.w = mes::pack_bf16x2(__uint_as_float(v[i + 6]) * inv, __uint_as_float(v[i + 7]) * inv);
        return o;
      };
      // A warp whose 32 rows all lie in the sequence stages each 64-column half of its rows
      // in shared memory (128-byte swizzle: 16-byte chunk c of row i at c ^ (i & 7)) and
      // writes it with one TMA store; a warp at the end of the sequence stores its valid
      // rows directly (a TMA box would also write the next sequence's rows).
      const int row0 = item.y * kTile + (warp & 3) * 32;
      if (row0 + 32 <= len) {
        uint8_t* stg = smem + kPOffStage + warp * kStageBytes;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          uint32_t v0[32], v1[32];
          mes::tmem_ld32(t_o + half * 64, v0);
          mes::tmem_ld32(t_o + half * 64 + 32, v1);
          if (o_stored) {  // the previous store must have read the staging block
            if (lane == 0) mes::tma_store_wait_read<0>();
            __syncwarp();
          }
          mes::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            *reinterpret_cast<uint4*>(stg + lane * 128 + ((c ^ (lane & 7)) * 16)) = scale8(v0, 8 * c);
            *reinterpret_cast<uint4*>(stg + lane * 128 + (((c + 4) ^ (lane & 7)) * 16)) = scale8(v1, 8 * c);
          }
          mes::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mes::tma_store_2d(&map_out, stg, h * kD + half * 64, start + row0);
            mes::tma_store_commit();
          }
          __syncwarp();
          o_stored = true;
        }
        mes::tc_fence_before();
        continue;
      }
      uint4* dst = reinterpret_cast<uint4*>(out + ((int64_t)(start + row_in_seq) * Hq + h) * kD);
      // Two 32-column buffers: the load of the next chunk is in flight while the current
      // one is scaled and stored, so only the first load's latency is exposed.
      auto store_chunk = [&](const uint32_t (&v)[32], int c) {
        if (!valid) return;
#pragma unroll
        for (int i = 0; i < 32; i += 8) dst[(c + i) / 8] = scale8(v, i);
      };
      {
        uint32_t v0[32], v1[32];
        mes::tmem_ld32(t_o + 0, v0);
        mes::tmem_wait_ld();
        mes::tmem_ld32(t_o + 32, v1);
        store_chunk(v0, 0);
        mes::tmem_wait_ld();
        mes::tmem_ld32(t_o + 64, v0);
        store_chunk(v1, 32);
        mes::tmem_wait_ld();
        mes::tmem_ld32(t_o + 96, v1);
        store_chunk(v0, 64);
        mes::tmem_wait_ld();
        store_chunk(v1, 96);
      }
      mes::tc_fence_before();
    }
    if (o_stored) {  // the staging blocks must outlive this warp's stores
      if (lane == 0) mes::tma_store_wait_all<0>();
      __syncwarp();
    }
  }

  mes::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    mes::tc_fence_after();
    mes::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

extern "C" int mes_attention_take_error(int* code) {
  int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_err_attn, sizeof(int));
  if (e != cudaSuccess) return MES_ERR_CUDA;
  e = cudaMemcpyToSymbol(g_err_attn, &zero, sizeof(int));
  *code = v;
  return mes_host::from_cuda(e);
}

// Element pairs (of every 8) whose exp2 runs on the FMA pipe in the head-pair kernel;
// MES_ATTN_POLY in {0, 2, 3, 4} overrides the default for measurements.
static int poly_pairs() {
  static const int v = [] {
    const char* e = getenv("MES_ATTN_POLY");
    const int x = e ? atoi(e) : 0;
    return (x == 2 || x == 3 || x == 4) ? x : 0;
  }();
  return v;
}

// L2 cache hints on the head-pair kernel's loads (K/V evict_last, Q evict_first);
// MES_ATTN_L2_HINTS=0 turns them off for measurements.
static int l2_hints() {
  static const int v = [] {
    const char* e = getenv("MES_ATTN_L2_HINTS");
    return (e && atoi(e) == 0) ? 0 : 1;
  }();
  return v;
}

// The head-pair kernel's register split must fit in what each SM sub-partition holds for
// the CTA at launch: three warps per sub-partition, one of them shrinking.
template <typename K>
static bool pair_kernel_registers_fit(K kern) {
  static std::atomic<int> fit{-1};  // the compiled register count is the same on every device
  int f = fit.load(std::memory_order_relaxed);
  if (f < 0) {
    cudaFuncAttributes a;
    if (cudaFuncGetAttributes(&a, kern) != cudaSuccess) return false;
    f = 3 * a.numRegs >= 2 * kSoftmaxRegs + kOtherRegs && a.maxThreadsPerBlock >= kPThreads;
    fit.store(f, std::memory_order_relaxed);
  }
  return f != 0;
}

// Workspace layout is defined next to mes_varlen_schedule (elementwise.cu).
extern "C" int64_t mes_varlen_workspace_size(int64_t T);

extern "C" int mes_varlen_attention(const void* qkv, int64_t ld, void* out, const void* workspace,
                                    int64_t T, int Hq, int Hkv, int D, float scale, void* stream) {
  if (D != kD || T <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv) return MES_ERR_INVALID;
  if (ld < (int64_t)(Hq + 2 * Hkv) * D || ld % 8 || T > 0x3fffffffLL) return MES_ERR_INVALID;
  if (!qkv || !out || !workspace) return MES_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255))
    return MES_ERR_ALIGN;
  CUtensorMap map;
  if (!mes_host::make_map_2d(&map, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, ld, ld, kTile, 64,
                             CU_TENSOR_MAP_SWIZZLE_128B))
    return MES_ERR_INVALID;
  const char* ws = static_cast<const char*>(workspace);
  const int64_t items_off = ((256 + 4 * (T + 1)) + 255) & ~int64_t(255);
  const int grid = mes_host::persistent_ctas();
  const float scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t s = (cudaStream_t)stream;
  const int poly = poly_pairs();
  auto kern = poly == 2   ? varlen_attention_pair_kernel<2>
              : poly == 3 ? varlen_attention_pair_kernel<3>
              : poly == 4 ? varlen_attention_pair_kernel<4>
                          : varlen_attention_pair_kernel<0>;
  if ((Hq / Hkv) % 2 == 0 && pair_kernel_registers_fit(kern)) {
    static std::atomic<uint64_t> attr_done[4];
    const int st = mes_host::once_per_device(attr_done[poly == 2 ? 1 : poly == 3 ? 2 : poly == 4 ? 3 : 0], [&] {
      return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem) == cudaSuccess
                 ? MES_OK : MES_ERR_CUDA;
    });
    if (st != MES_OK) return st;
    CUtensorMap map_out;
    if (!mes_host::make_map_2d(&map_out, out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, (int64_t)Hq * kD,
                               (int64_t)Hq * kD, 32, 64, CU_TENSOR_MAP_SWIZZLE_128B))
      return MES_ERR_INVALID;
    kern<<<grid, kPThreads, kPSmem, s>>>(map, map_out, (__nv_bfloat16*)out, (const int*)ws,
                                         (const int*)(ws + 256), (const int2*)(ws + items_off),
                                         Hq, Hkv, scale_log2, l2_hints());
    return mes_host::from_cuda(cudaGetLastError());
  }
  static std::atomic<uint64_t> attr_done1{0};
  const int st = mes_host::once_per_device(attr_done1, [] {
    return cudaFuncSetAttribute(varlen_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kSmem) == cudaSuccess ? MES_OK : MES_ERR_CUDA;
  });
  if (st != MES_OK) return st;
  varlen_attention_kernel<<<grid, kThreads, kSmem, s>>>(
      map, (__nv_bfloat16*)out, (const int*)ws, (const int*)(ws + 256), (const int2*)(ws + items_off),
      Hq, Hkv, scale_log2);
  return mes_host::from_cuda(cudaGetLastError());
}
