// Memory-bound kernels of the forward pass: embedding gather, RMSNorm, fused
// add+RMSNorm, fused per-head q/k RMSNorm + NeoX RoPE, SiLU-and-mul, last-token
// pooling + L2 normalisation, and the on-device varlen schedule.
//
// All of them move 16-byte vectors (8 bf16) with coalesced loads/stores and reduce with
// warp shuffles; statistics and transcendental math are fp32.
#include "common.cuh"

namespace {

__device__ int g_err_elementwise = 0;

using bf162 = __nv_bfloat162;

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const bf162* h = reinterpret_cast<const bf162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 v;
  uint32_t* u = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) u[i] = mes::pack_bf16x2(f[2 * i], f[2 * i + 1]);
  return v;
}
// 8 consecutive elements of a bf16 or fp32 row as fp32 registers.
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  unpack8(*reinterpret_cast<const uint4*>(p), f);
}
__device__ __forceinline__ void load8(const float* p, float (&f)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  *reinterpret_cast<uint4*>(p) = pack8(f);
}
__device__ __forceinline__ void store8(float* p, const float (&f)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

// Round fp32 to bf16 and back (the reference's `.to(orig_dtype)` before `* weight`).
__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum for blockDim.x <= 1024; every thread gets the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (l < nw) ? red[l] : 0.f;
  t = warp_sum(t);
  __syncthreads();
  return t;
}

// ------------------------------------ embedding ----------------------------------------
// out[t] = table[ids[t]] as bf16 (copy) or fp32 (exact widening, to start a fp32 residual).
template <typename OT>
__global__ void embedding_kernel(const int64_t* __restrict__ ids, int64_t T,
                                 const __nv_bfloat16* __restrict__ table, int64_t vocab, int64_t hv,
                                 OT* __restrict__ out) {
  const int64_t total = T * hv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / hv, c = i - t * hv;
    const int64_t id = __ldg(ids + t);
    float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (id >= 0 && id < vocab) {
      unpack8(__ldg(reinterpret_cast<const uint4*>(table + (id * hv + c) * 8)), f);
    } else if (c == 0) {
      atomicCAS(&g_err_elementwise, 0, MES_ERR_INVALID);
    }
    store8(out + i * 8, f);
  }
}

// ------------------------------------- RMSNorm -----------------------------------------
// One block per row, one 8-element vector per thread (blockDim.x = H / 8).  XT is the
// input type, RT the residual type (bf16: the reference's layout; fp32: the model's
// residual stream).  With kAdd, s = x + residual is formed in fp32, stored to
// residual_out (rounded to RT) and normalised; y = bf16(bf16(s * rsqrt(mean + eps)) * w).
template <typename XT, typename RT, bool kAdd>
__global__ void rmsnorm_kernel(const XT* x, const RT* residual, const uint4* __restrict__ w,
                               __nv_bfloat16* y, RT* residual_out, int hv, float inv_h, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int c = threadIdx.x;
  const int64_t off = (row * hv + c) * 8;
  float f[8];
  load8(x + off, f);
  if (kAdd) {
    float r[8];
    load8(residual + off, r);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] += r[i];
    store8(residual_out + off, f);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  ss = block_sum(ss, red);
  const float rs = rsqrtf(ss * inv_h + eps);
  float wf[8];
  unpack8(w[c], wf);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = round_bf16(f[i] * rs) * wf[i];
  store8(y + off, f);
}

// ------------------------------ q/k RMSNorm + NeoX RoPE --------------------------------
// 8 threads per (token, group of kGroupHeads heads): thread j owns elements 8j..8j+7 and
// 64+8j..64+8j+7 of each 128-wide head, so both elements that the NeoX rotate-half pairs are
// in the same thread (the rotation needs no shuffle) and a head's sum of squares takes three
// shuffles.  The token's cos/sin values (one set serves both halves) and the norm weights are
// loaded once per group, and the group's head loads are all in flight together
// (2 x kGroupHeads x 16 bytes per thread).  Units are token-major, so a block covers
// consecutive kilobytes of the packed qkv rows.  Two heads per unit keep the kernel at 64
// registers and four blocks (32 warps) per SM: measured at 20000 tokens x 24 heads, 4.8 TB/s
// against 4.5 TB/s for eight heads per unit at two blocks per SM.
constexpr int kGroupHeads = 2;
constexpr int kRopeMinBlocks = 4;
constexpr int kRopeThreads = 8;  // threads per unit
template <bool kF32Cache>
__device__ __forceinline__ void load_cos_sin(const void* cos_sin, int64_t ps, int cj, float (&c)[8],
                                             float (&s)[8]) {
  if (kF32Cache) {
    const float4* cs = reinterpret_cast<const float4*>(static_cast<const float*>(cos_sin) + ps * 128);
    const float4 a = __ldg(cs + cj / 4), b = __ldg(cs + cj / 4 + 1);
    const float4 d = __ldg(cs + 16 + cj / 4), e = __ldg(cs + 16 + cj / 4 + 1);
    c[0] = a.x; c[1] = a.y; c[2] = a.z; c[3] = a.w; c[4] = b.x; c[5] = b.y; c[6] = b.z; c[7] = b.w;
    s[0] = d.x; s[1] = d.y; s[2] = d.z; s[3] = d.w; s[4] = e.x; s[5] = e.y; s[6] = e.z; s[7] = e.w;
  } else {
    const uint4* cs = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(cos_sin) + ps * 128);
    unpack8(__ldg(cs + cj / 8), c);
    unpack8(__ldg(cs + 8 + cj / 8), s);
  }
}

template <bool kNorm, bool kF32Cache>
__global__ void __launch_bounds__(256, kRopeMinBlocks)
qknorm_rope_kernel(__nv_bfloat16* __restrict__ qkv, int64_t ld, const int64_t* __restrict__ pos,
                   const void* __restrict__ cos_sin, int64_t max_pos, const uint4* __restrict__ qw,
                   const uint4* __restrict__ kw, int T, int Hq, int Hkv, float eps) {
  const int nh = Hq + Hkv;
  const int ngroups = (nh + kGroupHeads - 1) / kGroupHeads;
  const int unit = blockIdx.x * (256 / kRopeThreads) + (threadIdx.x / kRopeThreads);
  const int j = threadIdx.x % kRopeThreads;
  const bool valid = unit < T * ngroups;
  const int t = valid ? unit / ngroups : 0;
  const int h0 = (unit - t * ngroups) * kGroupHeads;
  uint4* row = reinterpret_cast<uint4*>(qkv + (int64_t)t * ld) + h0 * 16 + j;
  uint4 lo[kGroupHeads], hi[kGroupHeads];
#pragma unroll
  for (int u = 0; u < kGroupHeads; ++u) {
    const bool live = valid && h0 + u < nh;
    lo[u] = live ? row[u * 16] : make_uint4(0, 0, 0, 0);
    hi[u] = live ? row[u * 16 + 8] : make_uint4(0, 0, 0, 0);
  }
  int64_t ps = valid ? __ldg(pos + t) : 0;
  if (ps < 0 || ps >= max_pos) {
    if (valid && j == 0 && h0 == 0) atomicCAS(&g_err_elementwise, 0, MES_ERR_INVALID);
    ps = 0;
  }
  float c[8], s[8];
  load_cos_sin<kF32Cache>(cos_sin, ps, j * 8, c, s);
  // Norm weights of this thread's two 8-element slices, for q heads and for k heads.
  uint4 wq_lo = make_uint4(0, 0, 0, 0), wq_hi = wq_lo, wk_lo = wq_lo, wk_hi = wq_lo;
  if (kNorm) {
    if (h0 < Hq) {
      wq_lo = __ldg(qw + j);
      wq_hi = __ldg(qw + 8 + j);
    }
    if (Hkv > 0 && h0 + kGroupHeads > Hq) {
      wk_lo = __ldg(kw + j);
      wk_hi = __ldg(kw + 8 + j);
    }
  }
#pragma unroll
  for (int u = 0; u < kGroupHeads; ++u) {
    // Every lane runs all the group's heads (the units of a warp may differ in head count
    // and the shuffles use the full mask); heads past the end compute on zeros and store
    // nothing.
    float a[8], b[8];
    unpack8(lo[u], a);
    unpack8(hi[u], b);
    if (kNorm) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += a[i] * a[i];
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += b[i] * b[i];
#pragma unroll
      for (int o = kRopeThreads / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rs = rsqrtf(ss * (1.0f / 128.0f) + eps);
      const bool is_q = h0 + u < Hq;
      float wa[8], wb[8];
      unpack8(is_q ? wq_lo : wk_lo, wa);
      unpack8(is_q ? wq_hi : wk_hi, wb);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        a[i] = round_bf16(round_bf16(a[i] * rs) * wa[i]);
        b[i] = round_bf16(round_bf16(b[i] * rs) * wb[i]);
      }
    }
    float oa[8], ob[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      oa[i] = a[i] * c[i] - b[i] * s[i];
      ob[i] = b[i] * c[i] + a[i] * s[i];
    }
    if (valid && h0 + u < nh) {
      row[u * 16] = pack8(oa);
      row[u * 16 + 8] = pack8(ob);
    }
  }
}

// ------------------------------------ SiLU-and-mul -------------------------------------
__global__ void silu_mul_kernel(const uint4* __restrict__ x, uint4* __restrict__ y,
                                int64_t rows, int64_t iv) {
  const int64_t total = rows * iv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / iv, c = i - r * iv;
    float g[8], u[8];
    unpack8(__ldg(x + r * 2 * iv + c), g);
    unpack8(__ldg(x + r * 2 * iv + iv + c), u);
#pragma unroll
    for (int k = 0; k < 8; ++k) g[k] = g[k] / (1.0f + expf(-g[k])) * u[k];
    y[i] = pack8(g);
  }
}

// ------------------------------ last token + L2 normalise ------------------------------
__global__ void last_token_l2_kernel(const uint4* __restrict__ hidden, int64_t T, int hv,
                                     const int64_t* __restrict__ idx, float4* __restrict__ out) {
  __shared__ float red[32];
  const int64_t b = blockIdx.x;
  int64_t t = __ldg(idx + b);
  const bool ok = t >= 0 && t < T;
  if (!ok) {
    if (threadIdx.x == 0) atomicCAS(&g_err_elementwise, 0, MES_ERR_INVALID);
    t = 0;
  }
  float ss = 0.f;
  float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int c = threadIdx.x; c < hv; c += blockDim.x) {
    unpack8(__ldg(hidden + t * hv + c), f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  ss = block_sum(ss, red);
  const float inv = ok ? 1.0f / fmaxf(sqrtf(ss), 1e-12f) : 0.f;
  for (int c = threadIdx.x; c < hv; c += blockDim.x) {
    unpack8(__ldg(hidden + t * hv + c), f);
    out[(b * hv + c) * 2] = make_float4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv);
    out[(b * hv + c) * 2 + 1] = make_float4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv);
  }
}

// -------------------------------- varlen schedule --------------------------------------
// Workspace layout (bytes): [0,4) num_seqs, [4,8) num_tile_items, [8,12) max_tiles,
// [256, 256 + 4(T+1)) cu_seqlens, then (aligned to 256) the tile items int2 {seq, qtile}
// ordered by descending qtile (longest causal rows first), capacity T + T/128 + 1.
constexpr int kSchedThreads = 1024;
constexpr int kQTile = 128;

__device__ __forceinline__ int block_excl_scan(int v, int* sm, int* total) {
  // Inclusive warp scan, then across warps.
  const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (l >= o) x += y;
  }
  if (l == 31) sm[w] = x;
  __syncthreads();
  if (w == 0) {
    int s = sm[l];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, s, o);
      if (l >= o) s += y;
    }
    sm[l] = s;
  }
  __syncthreads();
  const int before = (w > 0 ? sm[w - 1] : 0) + x - v;
  *total = sm[31];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(kSchedThreads)
varlen_schedule_kernel(const int64_t* __restrict__ pos, int T, int* __restrict__ hdr,
                       int* __restrict__ cu, int2* __restrict__ items) {
  __shared__ int sm[32];
  __shared__ int s_maxtiles;
  // Pass 1: sequence starts -> cu_seqlens.
  int base = 0;
  for (int c0 = 0; c0 < T; c0 += kSchedThreads) {
    const int i = c0 + threadIdx.x;
    int start = 0;
    if (i < T) start = (i == 0) || (pos[i] != pos[i - 1] + 1);
    int total;
    const int ex = block_excl_scan(start, sm, &total);
    if (start) cu[base + ex] = i;
    base += total;
  }
  const int B = base;
  if (threadIdx.x == 0) {
    cu[B] = T;
    hdr[0] = B;
    s_maxtiles = 0;
  }
  __syncthreads();
  // Pass 2: longest sequence in tiles.
  int mt = 0;
  for (int s = threadIdx.x; s < B; s += kSchedThreads)
    mt = max(mt, (cu[s + 1] - cu[s] + kQTile - 1) / kQTile);
  atomicMax(&s_maxtiles, mt);
  __syncthreads();
  const int J = s_maxtiles;
  // Pass 3: items ordered by descending tile index, sequences ascending within a tile.
  int n = 0;
  for (int j = J - 1; j >= 0; --j) {
    for (int c0 = 0; c0 < B; c0 += kSchedThreads) {
      const int s = c0 + threadIdx.x;
      int has = 0;
      if (s < B) has = (cu[s + 1] - cu[s] + kQTile - 1) / kQTile > j;
      int total;
      const int ex = block_excl_scan(has, sm, &total);
      if (has) items[n + ex] = make_int2(s, j);
      n += total;
    }
  }
  if (threadIdx.x == 0) {
    hdr[1] = n;
    hdr[2] = J;
  }
}

inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }
inline int64_t cu_offset() { return 256; }
inline int64_t items_offset(int64_t T) { return align256(cu_offset() + 4 * (T + 1)); }
inline int64_t items_capacity(int64_t T) { return T + T / kQTile + 1; }

inline int grid_for(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)mes_host::sm_count() * 32;
  if (b > cap) b = cap;
  return (int)(b < 1 ? 1 : b);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
inline bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }

}  // namespace

// =========================================================================================
// C ABI
// =========================================================================================
// One thread waits on a fresh mbarrier of arrival count 1 through the library's bounded
// wait (the one every pipeline role uses), arriving first when `arrive` is set.  Without the
// arrival the phase never completes: after `limit_ns` the wait gives up, raises the CTA's
// abort flag and records MES_ERR_TIMEOUT in the device error word, and the kernel returns.
__global__ void wait_probe_kernel(uint64_t limit_ns, int arrive) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  mes::mbar_init(&bar, 1);
  abort_flag = 0;
  mes::fence_barrier_init();
  if (arrive) mes::mbar_arrive(&bar);
  mes::mbar_wait_limit(&bar, 0, &abort_flag, &g_err_elementwise, MES_ERR_TIMEOUT, limit_ns);
}

extern "C" int mes_elementwise_take_error(int* code) {
  int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_err_elementwise, sizeof(int));
  if (e != cudaSuccess) return MES_ERR_CUDA;
  e = cudaMemcpyToSymbol(g_err_elementwise, &zero, sizeof(int));
  *code = v;
  return mes_host::from_cuda(e);
}

static int launch_embedding(bool f32, const int64_t* ids, int64_t T, const void* table,
                            int64_t vocab, int64_t H, void* out, void* stream) {
  if (T < 0 || vocab <= 0 || H <= 0 || H % 8) return MES_ERR_INVALID;
  if (T == 0) return MES_OK;
  if (!ids || !table || !out) return MES_ERR_INVALID;
  if (!aligned16(table) || !aligned16(out) || !aligned8(ids)) return MES_ERR_ALIGN;
  const int64_t hv = H / 8;
  cudaStream_t s = (cudaStream_t)stream;
  if (f32)
    embedding_kernel<float><<<grid_for(T * hv, 256), 256, 0, s>>>(
        ids, T, (const __nv_bfloat16*)table, vocab, hv, (float*)out);
  else
    embedding_kernel<__nv_bfloat16><<<grid_for(T * hv, 256), 256, 0, s>>>(
        ids, T, (const __nv_bfloat16*)table, vocab, hv, (__nv_bfloat16*)out);
  return mes_host::from_cuda(cudaGetLastError());
}

extern "C" int mes_embedding(const int64_t* ids, int64_t T, const void* table, int64_t vocab,
                             int64_t H, void* out, void* stream) {
  return launch_embedding(false, ids, T, table, vocab, H, out, stream);
}

extern "C" int mes_embedding_f32(const int64_t* ids, int64_t T, const void* table, int64_t vocab,
                                 int64_t H, float* out, void* stream) {
  return launch_embedding(true, ids, T, table, vocab, H, out, stream);
}

template <typename XT, typename RT, bool kAdd>
static int launch_rmsnorm(const void* x, const void* residual, const void* w, void* y,
                          void* residual_out, int64_t rows, int64_t H, float eps, void* stream) {
  if (rows < 0 || H <= 0 || H % 256 || H / 8 > 1024) return MES_ERR_INVALID;
  if (rows == 0) return MES_OK;
  if (!x || !w || !y || (kAdd && (!residual || !residual_out))) return MES_ERR_INVALID;
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) ||
      (kAdd && (!aligned16(residual) || !aligned16(residual_out))))
    return MES_ERR_ALIGN;
  if (rows > 0x7fffffffLL) return MES_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  const float inv_h = 1.0f / (float)H;
  const int hv = (int)(H / 8);
  rmsnorm_kernel<XT, RT, kAdd><<<(unsigned)rows, hv, 0, s>>>(
      (const XT*)x, (const RT*)residual, (const uint4*)w, (__nv_bfloat16*)y, (RT*)residual_out, hv,
      inv_h, eps);
  return mes_host::from_cuda(cudaGetLastError());
}

extern "C" int mes_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t H,
                           float eps, void* stream) {
  return launch_rmsnorm<__nv_bfloat16, __nv_bfloat16, false>(x, nullptr, w, y, nullptr, rows, H,
                                                             eps, stream);
}

extern "C" int mes_rmsnorm_f32in(const float* x, const void* w, void* y, int64_t rows, int64_t H,
                                 float eps, void* stream) {
  return launch_rmsnorm<float, float, false>(x, nullptr, w, y, nullptr, rows, H, eps, stream);
}

extern "C" int mes_add_rmsnorm(const void* x, const void* residual, const void* w, void* y,
                               void* residual_out, int64_t rows, int64_t H, float eps,
                               void* stream) {
  return launch_rmsnorm<__nv_bfloat16, __nv_bfloat16, true>(x, residual, w, y, residual_out, rows,
                                                            H, eps, stream);
}

extern "C" int mes_add_rmsnorm_f32res(const void* x, float* residual, const void* w, void* y,
                                      int64_t rows, int64_t H, float eps, void* stream) {
  return launch_rmsnorm<__nv_bfloat16, float, true>(x, residual, w, y, residual, rows, H, eps,
                                                    stream);
}

extern "C" int mes_qknorm_rope(void* qkv, int64_t ld, const int64_t* positions,
                               const void* cos_sin, int cos_sin_f32, int64_t max_pos,
                               const void* q_w, const void* k_w, int64_t T, int Hq, int Hkv,
                               int D, float eps, int apply_norm, void* stream) {
  if (D != 128 || T < 0 || Hq < 0 || Hkv < 0 || Hq + Hkv == 0 || max_pos <= 0) return MES_ERR_INVALID;
  if (ld < ((int64_t)Hq + Hkv) * D || ld % 8) return MES_ERR_INVALID;
  if (T == 0) return MES_OK;
  if (!qkv || !positions || !cos_sin) return MES_ERR_INVALID;
  if (apply_norm && ((Hq > 0 && !q_w) || (Hkv > 0 && !k_w))) return MES_ERR_INVALID;
  if (!aligned16(qkv) || !aligned16(cos_sin) || !aligned8(positions) ||
      (apply_norm && (!aligned16(q_w) || !aligned16(k_w))))
    return MES_ERR_ALIGN;
  const int64_t units = T * (((int64_t)Hq + Hkv + kGroupHeads - 1) / kGroupHeads);
  if (units > 0x7fffffffLL - 256) return MES_ERR_INVALID;
  const unsigned blocks = (unsigned)((units + 256 / kRopeThreads - 1) / (256 / kRopeThreads));
  cudaStream_t s = (cudaStream_t)stream;
  __nv_bfloat16* p = (__nv_bfloat16*)qkv;
  const uint4* qwp = (const uint4*)q_w;
  const uint4* kwp = (const uint4*)k_w;

  if (apply_norm) {
    if (cos_sin_f32)
      qknorm_rope_kernel<true, true><<<blocks, 256, 0, s>>>(p, ld, positions, cos_sin, max_pos, qwp, kwp, (int)T, Hq, Hkv, eps);
    else
      qknorm_rope_kernel<true, false><<<blocks, 256, 0, s>>>(p, ld, positions, cos_sin, max_pos, qwp, kwp, (int)T, Hq, Hkv, eps);
  } else {
    if (cos_sin_f32)
      qknorm_rope_kernel<false, true><<<blocks, 256, 0, s>>>(p, ld, positions, cos_sin, max_pos, nullptr, nullptr, (int)T, Hq, Hkv, eps);
    else
      qknorm_rope_kernel<false, false><<<blocks, 256, 0, s>>>(p, ld, positions, cos_sin, max_pos, nullptr, nullptr, (int)T, Hq, Hkv, eps);
  }
  return mes_host::from_cuda(cudaGetLastError());
}

extern "C" int mes_silu_mul(const void* x, void* y, int64_t rows, int64_t I, void* stream) {
  if (rows < 0 || I <= 0 || I % 8) return MES_ERR_INVALID;
  if (rows == 0) return MES_OK;
  if (!x || !y) return MES_ERR_INVALID;
  if (!aligned16(x) || !aligned16(y)) return MES_ERR_ALIGN;
  const int64_t iv = I / 8;
  silu_mul_kernel<<<grid_for(rows * iv, 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint4*)x, (uint4*)y, rows, iv);
  return mes_host::from_cuda(cudaGetLastError());
}

extern "C" int mes_last_token_l2(const void* hidden, int64_t T, int64_t H, const int64_t* idx,
                                 int64_t B, float* out, void* stream) {
  if (T < 0 || H <= 0 || H % 8 || B < 0) return MES_ERR_INVALID;
  if (B == 0) return MES_OK;
  if (!hidden || !idx || !out || T == 0) return MES_ERR_INVALID;
  if (!aligned16(hidden) || !aligned16(out) || !aligned8(idx)) return MES_ERR_ALIGN;
  const int hv = (int)(H / 8);
  const int threads = hv >= 256 ? 256 : ((hv + 31) / 32) * 32;
  last_token_l2_kernel<<<(unsigned)B, threads, 0, (cudaStream_t)stream>>>(
      (const uint4*)hidden, T, hv, idx, (float4*)out);
  return mes_host::from_cuda(cudaGetLastError());
}

extern "C" int64_t mes_varlen_workspace_size(int64_t T) {
  if (T < 0) return -1;
  return items_offset(T) + 8 * items_capacity(T);
}

extern "C" int mes_varlen_schedule(const int64_t* positions, int64_t T, void* workspace,
                                   void* stream) {
  if (T <= 0 || T > 0x3fffffffLL || !positions || !workspace) return MES_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) || !aligned8(positions)) return MES_ERR_ALIGN;
  char* ws = static_cast<char*>(workspace);
  varlen_schedule_kernel<<<1, kSchedThreads, 0, (cudaStream_t)stream>>>(
      positions, (int)T, (int*)ws, (int*)(ws + cu_offset()), (int2*)(ws + items_offset(T)));
  return mes_host::from_cuda(cudaGetLastError());
}

extern "C" int mes_varlen_cu_seqlens(const void* workspace, int64_t T, int32_t* cu_seqlens,
                                     int32_t* num_seqs, void* stream) {
  if (T <= 0 || !workspace || !cu_seqlens || !num_seqs) return MES_ERR_INVALID;
  const char* ws = static_cast<const char*>(workspace);
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(cu_seqlens, ws + cu_offset(), 4 * (T + 1),
                                  cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(num_seqs, ws, 4, cudaMemcpyDeviceToDevice, s);
  return mes_host::from_cuda(e);
}

extern "C" int mes_wait_probe(int64_t limit_ns, int arrive, void* stream) {
  if (limit_ns <= 0 || limit_ns > 100000000) return MES_ERR_INVALID;  // at most 100 ms
  wait_probe_kernel<<<1, 1, 0, (cudaStream_t)stream>>>((uint64_t)limit_ns, arrive ? 1 : 0);
  return mes_host::from_cuda(cudaGetLastError());
}
