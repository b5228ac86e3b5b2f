// Varlen causal attention for callers that cannot allocate device memory.
//
// mes_varlen_attention needs a scratch workspace (cu_seqlens, sequence count and the
// query-tile work list written by mes_varlen_schedule) that the caller allocates.  Some
// callers have no way to do that: a host runtime that binds this library through a thin
// FFI and only holds the input and output buffers its tensor framework handed over, or a
// serving process whose device memory is carved up in advance by its own pool and may
// not grow while a request is in flight.  For them, mes_varlen_attention_noalloc keeps
// the workspace in a fixed array compiled into this library instead.
//
// The array lives on every GPU that loads the library, for as long as the process runs
// (kNoAllocMaxTokens tokens -> about 1.5 MiB).  All calls on a device share it and it
// keeps whatever the last call wrote; the schedule step rewrites every word the attention
// step reads, so nothing has to be cleared between calls.  Two calls whose GPU work
// overlaps (different streams, no ordering between them) race on the array.
#include <mutex>

#include "common.cuh"

namespace {

// Largest packed batch (tokens) the fixed workspace holds.
constexpr int64_t kNoAllocMaxTokens = 131072;

// Byte size of the schedule workspace for T tokens: header (256 B), cu_seqlens (i32 T+1,
// rounded up to 256 B), then the (sequence, query tile) items (8 B each, T + T/128 + 1).
constexpr int64_t workspace_bytes(int64_t T) {
  return ((256 + 4 * (T + 1) + 255) / 256) * 256 + 8 * (T + T / 128 + 1);
}

static __device__ __align__(256) unsigned char g_noalloc_workspace[workspace_bytes(kNoAllocMaxTokens)];

// Device address of g_noalloc_workspace, cached per device together with the CUDA context
// it was looked up in.  In host code the symbol's name is only a stand-in, so the address is
// looked up with that device current: on the first call in a context (the primary context,
// or one a caller created itself) and again whenever the current context of the device has
// changed, for instance after cudaDeviceReset created a new primary context.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
constexpr int kMaxDevices = 64;
struct WorkspaceAddr {
  CUcontext ctx;
  void* ptr;
};
WorkspaceAddr g_workspace[kMaxDevices] = {};
std::mutex g_workspace_mu;

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

int workspace_for_current_device(void** ptr) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MES_ERR_CUDA;
  CtxGetCurrentFn get_ctx = ctx_get_current_fn();
  CUcontext ctx = nullptr;
  if (!get_ctx || get_ctx(&ctx) != CUDA_SUCCESS) return MES_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_workspace_mu);
  WorkspaceAddr& w = g_workspace[dev];
  if (ctx != nullptr && w.ptr != nullptr && w.ctx == ctx) {
    *ptr = w.ptr;
    return MES_OK;
  }
  // The lookup binds the device's primary context to this thread when it had none, so the
  // context is read again afterwards.
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_workspace) != cudaSuccess || p == nullptr)
    return MES_ERR_CUDA;
  if (get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) return MES_ERR_CUDA;
  w.ctx = ctx;
  w.ptr = p;
  *ptr = p;
  return MES_OK;
}

}  // namespace

extern "C" int64_t mes_varlen_workspace_size(int64_t T);
extern "C" int mes_varlen_schedule(const int64_t* positions, int64_t T, void* workspace,
                                   void* stream);
extern "C" int mes_varlen_attention(const void* qkv, int64_t ld, void* out, const void* workspace,
                                    int64_t T, int Hq, int Hkv, int D, float scale, void* stream);

extern "C" int64_t mes_varlen_attention_noalloc_max_tokens(void) { return kNoAllocMaxTokens; }

extern "C" int mes_varlen_attention_noalloc(const int64_t* positions, const void* qkv, int64_t ld,
                                            void* out, int64_t T, int Hq, int Hkv, int D,
                                            float scale, void* stream) {
  if (T <= 0 || T > kNoAllocMaxTokens) return MES_ERR_INVALID;
  if (mes_varlen_workspace_size(T) > workspace_bytes(kNoAllocMaxTokens)) return MES_ERR_INVALID;
  void* ws = nullptr;
  const int st = workspace_for_current_device(&ws);
  if (st != MES_OK) return st;
  const int s1 = mes_varlen_schedule(positions, T, ws, stream);
  if (s1 != MES_OK) return s1;
  return mes_varlen_attention(qkv, ld, out, ws, T, Hq, Hkv, D, scale, stream);
}
