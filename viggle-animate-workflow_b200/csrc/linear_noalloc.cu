// slim_int8_linear_noalloc: the convrot linear for callers that cannot allocate device
// memory.
//
// Who needs it: code that runs inside a host framework whose device memory it does not own
// (a plugin handed only the input/output buffers by an engine with its own pool), code on a
// path where a cudaMalloc would synchronise the device or fail under a memory cap, and code
// that must not grow its footprint between calls. slim_int8_linear asks the caller for two
// workspaces (the per-token int8 codes and scales of the activation); this variant keeps
// them in a fixed array compiled into the library instead.
//
// The scratch is one file-scope device array of kNoAllocScratchBytes (32 MiB). Every GPU on
// which the library's module is loaded holds those 32 MiB until the process exits. A call
// needs round_up(M*K, 256) + 4*M bytes of it (codes, then scales); larger calls are
// rejected with SLIM_ERR_SHAPE.
//
// The array's device address is looked up once per device and CUDA context, on the first call
// made with that device and context current (cudaGetSymbolAddress; the host-side name of the
// array is only a stand-in and is never given to a kernel), and looked up again when the
// current context changes (a caller's own driver context, or a new primary context after a
// device reset). Make the first call in a context before any stream capture.
//
// Every call shares the array, and it keeps the previous call's contents. Nothing in it
// needs to start at zero: the activation quantiser writes every code and scale that the
// GEMM then reads. Calls that overlap on the GPU (concurrent streams, or threads issuing on
// different streams) race on the array; serialise them on one stream.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/slimdit_b200.h"
#include "slim_kernels.h"

namespace slim {

constexpr size_t kNoAllocScratchBytes = size_t{32} << 20;

static __device__ __align__(256) unsigned char g_linear_scratch[kNoAllocScratchBytes];

static std::mutex g_scratch_mu;
static void* g_scratch_addr[64] = {nullptr};
static CUcontext g_scratch_ctx[64] = {nullptr};

// The calling thread's current driver context, through the runtime's driver entry point (the
// library does not link the driver library itself).
static int current_context(CUcontext* ctx) {
  using GetCurrent = CUresult (*)(CUcontext*);
  static GetCurrent get_current = nullptr;
  if (get_current == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult found = cudaDriverEntryPointSymbolNotFound;
    const cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &found);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDriverEntryPoint(cuCtxGetCurrent)");
    if (found != cudaDriverEntryPointSuccess || fn == nullptr) return fail(SLIM_ERR_CUDA, "cuCtxGetCurrent not found");
    get_current = reinterpret_cast<GetCurrent>(fn);
  }
  if (get_current(ctx) != CUDA_SUCCESS) return fail(SLIM_ERR_CUDA, "cuCtxGetCurrent failed");
  return SLIM_OK;
}

// Device address of g_linear_scratch in the current device's current context, looked up once per
// device and context.
static int linear_scratch_address(void** addr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(SLIM_ERR_ARCH, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  CUcontext ctx = nullptr;
  int rc = current_context(&ctx);
  if (rc != SLIM_OK) return rc;
  if (g_scratch_addr[dev] == nullptr || ctx == nullptr || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_linear_scratch);  // makes the primary context current if none is
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(linear scratch)");
    if (p == nullptr) return fail(SLIM_ERR_CUDA, "linear scratch has no device address");
    if ((rc = current_context(&ctx)) != SLIM_OK) return rc;
    g_scratch_addr[dev] = p;
    g_scratch_ctx[dev] = ctx;
  }
  *addr = g_scratch_addr[dev];
  return SLIM_OK;
}

}  // namespace slim

extern "C" int slim_int8_linear_noalloc(const void* x, int x_dtype, const int8_t* qw, const float* sw,
                                        const void* bias, void* out, int64_t M, int64_t N, int64_t K,
                                        int group, int epilogue, void* stream) {
  using namespace slim;
  SLIM_NVTX("slim_int8_linear_noalloc");
  int rc;
  if ((rc = check_group(K, group)) != SLIM_OK) return rc;
  if ((rc = check_dtype(x_dtype)) != SLIM_OK) return rc;
  if (K > 16384) return fail(SLIM_ERR_SHAPE, "in_features above 16384 not supported by the activation quantiser");
  if (M < 0 || N <= 0) return fail(SLIM_ERR_SHAPE, "bad shape M=%lld N=%lld", static_cast<long long>(M), static_cast<long long>(N));
  if (M > (int64_t{1} << 31)) return fail(SLIM_ERR_SHAPE, "M=%lld too large", static_cast<long long>(M));
  const int64_t code_bytes = (M * K + 255) / 256 * 256;
  const int64_t need = code_bytes + 4 * M;
  if (need > static_cast<int64_t>(kNoAllocScratchBytes))
    return fail(SLIM_ERR_SHAPE,
                "M*K=%lld needs %lld scratch bytes; the allocation-free linear has %lld (round_up(M*K,256) + 4*M must fit)",
                static_cast<long long>(M * K), static_cast<long long>(need), static_cast<long long>(kNoAllocScratchBytes));
  if (M == 0) return SLIM_OK;
  if (x == nullptr) return fail(SLIM_ERR_NULL, "x is NULL");
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0) return fail(SLIM_ERR_ALIGN, "x must be 16-byte aligned");
  if ((rc = check_arch()) != SLIM_OK) return rc;
  void* scratch = nullptr;
  if ((rc = linear_scratch_address(&scratch)) != SLIM_OK) return rc;
  int8_t* xq = static_cast<int8_t*>(scratch);
  float* sx = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + code_bytes);
  if ((rc = gemm_checks(xq, qw, sx, sw, bias, out, nullptr, M, N, K, epilogue)) != SLIM_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_act_quant(x, x_dtype, M, static_cast<int>(K), xq, sx, st);
  if (e != cudaSuccess) return cuda_fail(e, "activation quant launch");
  note_launch();
  GemmI8Params p{xq, qw, sx, sw, bias, out, nullptr, M, N, K, out_pitch(N, epilogue), epilogue};
  e = launch_gemm_i8(p, st);
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  note_launch();
  return SLIM_OK;
}
