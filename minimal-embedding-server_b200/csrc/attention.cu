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
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 1);
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
      int n_item = 0, kvit = 0;
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
        // Give copies already in flight time to land before the CTA exits.
        const uint64_t t = mes::globaltimer_ns();
        while (mes::globaltimer_ns() - t < 1000000ull) {
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
        const uint64_t t = mes::globaltimer_ns();
        while (mes::globaltimer_ns() - t < 1000000ull) {
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

}  // namespace

extern "C" int mes_attention_take_error(int* code) {
  int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_err_attn, sizeof(int));
  if (e != cudaSuccess) return MES_ERR_CUDA;
  e = cudaMemcpyToSymbol(g_err_attn, &zero, sizeof(int));
  *code = v;
  return mes_host::from_cuda(e);
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
  cudaError_t e = cudaFuncSetAttribute(varlen_attention_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) return MES_ERR_CUDA;
  const char* ws = static_cast<const char*>(workspace);
  const int64_t items_off = ((256 + 4 * (T + 1)) + 255) & ~int64_t(255);
  const int grid = mes_host::sm_count();
  varlen_attention_kernel<<<grid, kThreads, kSmem, (cudaStream_t)stream>>>(
      map, (__nv_bfloat16*)out, (const int*)ws, (const int*)(ws + 256), (const int2*)(ws + items_off),
      Hq, Hkv, scale * 1.4426950408889634f);
  return mes_host::from_cuda(cudaGetLastError());
}
