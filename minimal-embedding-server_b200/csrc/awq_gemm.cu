// AWQ W4A16 GEMM on tcgen05 / TMEM, plus the load-time repack and a standalone
// dequantiser that shares the GEMM's arithmetic.
//
// Y[M, N] = X[M, K] * W[K, N] (+ bias), W[k, n] = bf16_rne((q - z) * s).
//
// The product is computed transposed, Y^T = W^T X^T, so that the weights are the MMA's
// A operand and can live in tensor memory:
//   * a TMA warp streams X tiles (BT tokens x 64 k, bf16, 128-byte swizzle) and the packed
//     weight tile (8 words x 128 features of the kernel layout) into a ring of smem stages;
//   * four dequant warps (one per TMEM lane quadrant, one output feature per thread) turn
//     8 words = 64 k of their feature into 32 bf16x2 registers and write them with
//     tcgen05.st into the stage's TMEM A slot - the bf16 weights never touch smem or HBM;
//   * one thread issues tcgen05.mma (M = 128 features, N = BT tokens, K = 16) reading A from
//     TMEM and B (= X) from smem, accumulating fp32 in TMEM, and frees each stage with
//     tcgen05.commit;
//   * the same four warps drain the accumulator (tcgen05.ld), add the bias, convert to bf16
//     and write 32x32 blocks through smem with TMA stores.
//
// Exact dequantisation in bf16x2 arithmetic: the code pair (q_k, q_k+1) is extracted as the
// bf16 pair (128 + q) with one LOP3 (the nibble interleave puts k and k+1 at bits 4j and
// 16 + 4j); subtracting (128 + z) is exact; the fp16 scale is split into s_hi = bf16(s) and
// s_lo = bf16(s - s_hi) (exact, <= 3 significant bits), (q - z) * s_lo is exact in bf16,
// and fma.rn(q - z, s_hi, (q - z) * s_lo) rounds (q - z) * s exactly once.
#include "common.cuh"

namespace {

__device__ int g_err_gemm = 0;

constexpr int kBN = 128;  // output features per tile (MMA M)
constexpr int kBK = 64;   // k per pipeline stage (one 128-byte swizzle row of bf16)
constexpr int kGroup = 128;
constexpr int kThreads = 192;  // warp 0 TMA, warp 1 MMA + TMEM alloc, warps 2..5 dequant/epilogue

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
template <int BT, int STAGES>
struct Cfg {
  static constexpr int kXStage = BT * kBK * 2;
  static constexpr int kWStage = (kBK / 8) * kBN * 4;
  static constexpr int kOutBuf = 32 * 32 * 2;
  static constexpr int kOffX = 0;
  static constexpr int kOffW = STAGES * kXStage;
  static constexpr int kOffOut = kOffW + STAGES * kWStage;
  static constexpr int kOffBar = kOffOut + 4 * 2 * kOutBuf;
  static constexpr int kSmem = kOffBar + 256 + 1024;  // barriers + 1 KB alignment slack
  static constexpr int kChunk = BT < 32 ? BT : 32;  // tokens per epilogue store
  static constexpr int kTmemNeed = BT + STAGES * 32;
  static constexpr int kTmemCols = kTmemNeed <= 32 ? 32 : kTmemNeed <= 64 ? 64
                                 : kTmemNeed <= 128 ? 128 : kTmemNeed <= 256 ? 256 : 512;
  static_assert(kTmemNeed <= 512, "TMEM budget");
  static_assert(BT % 16 == 0 && BT >= 16 && BT <= 256, "MMA N");
  static_assert(kXStage % 1024 == 0, "swizzle atoms");
};

// kResidual: instead of storing bf16 Y, the epilogue accumulates into a fp32 residual
// stream, R[t, n] += acc + bias (the residual add of the decoder block fused into the
// o_proj / down_proj GEMM).
template <int BT, int STAGES, bool kResidual>
__global__ void __launch_bounds__(kThreads)
awq_gemm_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                const __grid_constant__ CUtensorMap map_y, const int32_t* __restrict__ qzeros,
                const uint16_t* __restrict__ scales, const __nv_bfloat16* __restrict__ bias,
                float* __restrict__ R, int64_t ldr, int M, int N, int K) {
  using C = Cfg<BT, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem + C::kOffX;
  const uint32_t* ws = reinterpret_cast<const uint32_t*>(smem + C::kOffW);
  __nv_bfloat16* outbuf = reinterpret_cast<__nv_bfloat16*>(smem + C::kOffOut);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* full = bars;                  // TMA landed (X + W words)
  uint64_t* afull = bars + STAGES;        // dequantised A written to TMEM
  uint64_t* empty = bars + 2 * STAGES;    // MMAs of the stage done
  uint64_t* accum = bars + 3 * STAGES;    // all MMAs done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = mes::warp_id(), lane = mes::lane_id();
  const int n0 = blockIdx.x * kBN;
  const int t0 = blockIdx.y * BT;
  const int nk = K / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mes::mbar_init(&full[s], 1);
      mes::mbar_init(&afull[s], 4);
      mes::mbar_init(&empty[s], 1);
    }
    mes::mbar_init(accum, 1);
    *abort_flag = 0;
    mes::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    mes::tma_prefetch_desc(&map_x);
    mes::tma_prefetch_desc(&map_w);
    mes::tma_prefetch_desc(&map_y);
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
  const uint32_t tmem_a = tmem + BT;  // A stages after the BT accumulator columns

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------------
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES;
        if (kb >= STAGES &&
            !mes::mbar_wait(&empty[s], ((kb / STAGES) & 1) ^ 1, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT))
          break;
        mes::mbar_arrive_expect_tx(&full[s], C::kXStage + C::kWStage);
        mes::tma_load_2d(xs + s * C::kXStage, &map_x, &full[s], kb * kBK, t0);
        mes::tma_load_2d((void*)(ws + s * (C::kWStage / 4)), &map_w, &full[s], n0, kb * (kBK / 8));
        issued = kb + 1;
      }
      if (*abort_flag) {
        // Let the copies already issued land before the CTA exits.
        for (int kb = issued - STAGES < 0 ? 0 : issued - STAGES; kb < issued; ++kb) {
          const uint64_t tstart = mes::globaltimer_ns();
          while (!mes::mbar_try_wait(&full[kb % STAGES], (kb / STAGES) & 1) &&
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
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mes::mbar_wait(&full[s], ph, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT)) break;
        if (!mes::mbar_wait(&afull[s], ph, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT)) break;
        mes::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t bdesc =
              mes::smem_desc_sw128(xs_addr + s * C::kXStage + kk * 32, 16, 1024);
          mes::mma_ts(tmem, tmem_a + s * 32 + kk * 8, bdesc, idesc, (kb | kk) != 0);
        }
        mes::tc_commit(&empty[s]);
      }
      mes::tc_commit(accum);
      if (*abort_flag) {
        const uint64_t tstart = mes::globaltimer_ns();
        while (!mes::mbar_try_wait(accum, 0) && mes::globaltimer_ns() - tstart < mes::kWaitLimitNs) {
        }
      }
    }
    __syncwarp();
  } else {
    // --------------------------- dequant + epilogue warps -----------------------------
    const int q = warp & 3;                 // TMEM lane quadrant of this warp
    const int row = q * 32 + lane;          // feature within the tile
    const int n = n0 + row;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int zshift = 4 * kInvOrder[n & 7];
    const int NW = N >> 3;
    // Group parameters: raw values of the next group are loaded one group ahead.
    uint32_t zraw = __ldg(qzeros + (n >> 3));
    uint16_t sraw = __ldg(scales + n);
    GroupParams gp = make_group(zraw, zshift, sraw);
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % STAGES;
      const uint32_t ph = (kb / STAGES) & 1;
      if ((kb & 1) == 0) {  // a new 128-wide group starts every other stage
        gp = make_group(zraw, zshift, sraw);
        const int gn = (kb >> 1) + 1;
        if (gn < K / kGroup) {
          zraw = __ldg(qzeros + (int64_t)gn * NW + (n >> 3));
          sraw = __ldg(scales + (int64_t)gn * N + n);
        }
      }
      if (!mes::mbar_wait_warp(&full[s], ph, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT)) { ok = false; break; }
      mes::tc_fence_after();
      const uint32_t* wsrc = ws + s * (C::kWStage / 4) + row;
      uint32_t a[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t w = wsrc[i * kBN];
        a[4 * i + 0] = dq_pair(w, gp);
        a[4 * i + 1] = dq_pair(w >> 4, gp);
        a[4 * i + 2] = dq_pair(w >> 8, gp);
        a[4 * i + 3] = dq_pair(w >> 12, gp);
      }
      mes::tmem_st32(tmem_a + s * 32 + lane_off, a);
      mes::tmem_wait_st();
      mes::tc_fence_before();
      __syncwarp();
      if (lane == 0) mes::mbar_arrive(&afull[s]);
      __syncwarp();
    }
    if (ok && mes::mbar_wait_warp(accum, 0, abort_flag, &g_err_gemm, MES_ERR_TIMEOUT)) {
      mes::tc_fence_after();
      const float b = bias ? __bfloat162float(bias[n]) : 0.f;
      __nv_bfloat16* mybuf = outbuf + (warp - 2) * 2 * 32 * 32;
#pragma unroll 1
      for (int c0 = 0; c0 < BT; c0 += C::kChunk) {
        uint32_t v[C::kChunk];
        if constexpr (C::kChunk == 32) mes::tmem_ld32(tmem + lane_off + c0, v);
        else mes::tmem_ld16(tmem + lane_off + c0, v);
        mes::tmem_wait_ld();
        if (t0 + c0 >= M) break;  // rows past the end of X: nothing to store
        if constexpr (kResidual) {
          // Each lane owns feature n; a warp touches 32 consecutive fp32 per token row.
          const int rows = min(C::kChunk, M - (t0 + c0));
          float* rp = R + (int64_t)(t0 + c0) * ldr + n;
          float rv[C::kChunk];
#pragma unroll
          for (int j = 0; j < C::kChunk; ++j) rv[j] = j < rows ? rp[(int64_t)j * ldr] : 0.f;
#pragma unroll
          for (int j = 0; j < C::kChunk; ++j)
            if (j < rows) rp[(int64_t)j * ldr] = rv[j] + (__uint_as_float(v[j]) + b);
        } else {
          __nv_bfloat16* buf = mybuf + ((c0 / C::kChunk) & 1) * 32 * 32;
          if (c0 >= 2 * C::kChunk) {
            if (lane == 0) mes::tma_store_wait_read<1>();
            __syncwarp();
          }
#pragma unroll
          for (int j = 0; j < C::kChunk; ++j)
            buf[j * 32 + lane] = __float2bfloat16_rn(__uint_as_float(v[j]) + b);
          mes::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mes::tma_store_2d(&map_y, buf, n0 + q * 32, t0 + c0);
            mes::tma_store_commit();
          }
          __syncwarp();
        }
      }
      if (lane == 0) mes::tma_store_wait_all<0>();
      __syncwarp();
    }
  }

  mes::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    mes::tc_fence_after();
    mes::tmem_dealloc(tmem, C::kTmemCols);
  }
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

template <int BT, int STAGES, bool kResidual>
int launch_gemm(const void* X, int64_t ldx, const int32_t* qw, const int32_t* qzeros,
                const void* scales, const void* bias, void* Y, int64_t ldy, int64_t M,
                int64_t N, int64_t K, cudaStream_t stream) {
  using C = Cfg<BT, STAGES>;
  cudaError_t e = cudaFuncSetAttribute(awq_gemm_kernel<BT, STAGES, kResidual>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  if (e != cudaSuccess) return MES_ERR_CUDA;
  CUtensorMap mx, mw, my;
  if (!mes_host::make_map_2d(&mx, X, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, ldx, BT, kBK,
                             CU_TENSOR_MAP_SWIZZLE_128B) ||
      !mes_host::make_map_2d(&mw, qw, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, K / 8, N, N, kBK / 8, kBN,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
    return MES_ERR_INVALID;
  if (kResidual) {
    my = mx;  // unused by the residual epilogue
  } else if (!mes_host::make_map_2d(&my, Y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, N, ldy,
                                    C::kChunk, 32, CU_TENSOR_MAP_SWIZZLE_NONE)) {
    return MES_ERR_INVALID;
  }
  dim3 grid((unsigned)(N / kBN), (unsigned)((M + BT - 1) / BT));
  awq_gemm_kernel<BT, STAGES, kResidual><<<grid, kThreads, C::kSmem, stream>>>(
      mx, mw, my, qzeros, (const uint16_t*)scales, (const __nv_bfloat16*)bias,
      kResidual ? (float*)Y : nullptr, ldy, (int)M, (int)N, (int)K);
  return mes_host::from_cuda(cudaGetLastError());
}

template <bool kResidual>
int dispatch_gemm(const void* X, int64_t ldx, const int32_t* qw, const int32_t* qzeros,
                  const void* scales, const void* bias, void* Y, int64_t ldy, int64_t M,
                  int64_t N, int64_t K, cudaStream_t s) {
  if (M <= 16) return launch_gemm<16, 6, kResidual>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
  if (M <= 32) return launch_gemm<32, 6, kResidual>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
  if (M <= 64) return launch_gemm<64, 6, kResidual>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
  return launch_gemm<128, 4, kResidual>(X, ldx, qw, qzeros, scales, bias, Y, ldy, M, N, K, s);
}

int check_gemm_args(const void* X, int64_t ldx, const int32_t* qw, const int32_t* qzeros,
                    const void* scales, const void* Y, int64_t ldy, int64_t M, int64_t N,
                    int64_t K, int group_size, int y_elem_align) {
  if (M < 0 || N <= 0 || K <= 0 || N % kBN || K % kGroup || group_size != kGroup)
    return MES_ERR_INVALID;
  if (N > (1 << 30) || K > (1 << 30) || M > (1LL << 31) - 256) return MES_ERR_INVALID;
  if (ldx < K || ldy < N || ldx % 8 || ldy % y_elem_align) return MES_ERR_INVALID;
  if (M == 0) return -1;
  if (!X || !qw || !qzeros || !scales || !Y) return MES_ERR_INVALID;
  return MES_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

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
  if (!aligned16(w_out)) return MES_ERR_ALIGN;
  const int64_t total = (K / 8) * N;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 65535) blocks = 65535;
  awq_dequant_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      (const uint32_t*)qweight_mes, qzeros, (const uint16_t*)scales, K, N, (uint4*)w_out);
  return mes_host::from_cuda(cudaGetLastError());
}

extern "C" int mes_awq_gemm(const void* X, int64_t ldx, const int32_t* qweight_mes,
                            const int32_t* qzeros, const void* scales, const void* bias, void* Y,
                            int64_t ldy, int64_t M, int64_t N, int64_t K, int group_size,
                            void* stream) {
  const int st = check_gemm_args(X, ldx, qweight_mes, qzeros, scales, Y, ldy, M, N, K,
                                 group_size, 8);
  if (st != MES_OK) return st < 0 ? MES_OK : st;
  if (!aligned16(X) || !aligned16(Y) || !aligned16(qweight_mes)) return MES_ERR_ALIGN;
  return dispatch_gemm<false>(X, ldx, qweight_mes, qzeros, scales, bias, Y, ldy, M, N, K,
                              (cudaStream_t)stream);
}

extern "C" int mes_awq_gemm_residual(const void* X, int64_t ldx, const int32_t* qweight_mes,
                                     const int32_t* qzeros, const void* scales, const void* bias,
                                     float* R, int64_t ldr, int64_t M, int64_t N, int64_t K,
                                     int group_size, void* stream) {
  const int st = check_gemm_args(X, ldx, qweight_mes, qzeros, scales, R, ldr, M, N, K,
                                 group_size, 1);
  if (st != MES_OK) return st < 0 ? MES_OK : st;
  if (!aligned16(X) || !aligned16(qweight_mes) || (reinterpret_cast<uintptr_t>(R) & 3))
    return MES_ERR_ALIGN;
  return dispatch_gemm<true>(X, ldx, qweight_mes, qzeros, scales, bias, R, ldr, M, N, K,
                             (cudaStream_t)stream);
}
