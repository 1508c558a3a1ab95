// ttn_select_f16_static: YOLO26 detection selection for callers that cannot
// allocate device memory.
//
// Some hosts of this library have no device allocator to hand: bindings that
// only see raw pointers handed to them by another runtime (a JNI/cgo-style
// shim, an inference server plugin whose framework owns every device byte), or
// real-time loops that forbid allocation after start-up.  ttn_select_f16 needs
// caller-provided scratch; this variant uses a fixed scratch array compiled into
// the library instead, so the caller passes only the input and output buffers.
//
// Limits and sharing:
//  * the scratch array holds kStaticScratchBytes (8 MiB) -- enough for e.g. 64
//    images of 8400 anchors x 80 classes at max_det 300 -- and every GPU that
//    loads the library keeps it until the process exits;
//  * larger requests are rejected with TTN_UNSUPPORTED before anything runs;
//  * every call shares the one array per device, and calls whose kernels overlap
//    on the GPU (different streams, no ordering between them) race on it; calls
//    on one stream are ordered and safe;
//  * the array keeps the previous call's contents: the selection kernels write
//    every scratch word they read, so nothing has to start at zero;
//  * the array's device address belongs to the CUDA context current on the
//    calling thread (the device's primary context, or a context the host made
//    with the driver API).  Outside stream capture every call looks it up afresh
//    with cudaGetSymbolAddress (a host-side lookup that allocates nothing), so a
//    context created later, or re-created by cudaDeviceReset, gets its own
//    address; the lookup is remembered per context.  Under stream capture no
//    lookup is made: the address remembered for the current context is used,
//    and if there is none (no call yet outside capture in this context) the call
//    is rejected with TTN_INVALID_ARG -- make one call outside capture first.
// The entry point itself calls no cudaMalloc, cudaFree or other allocating
// routine.
#include <cuda.h>  // CUcontext / CUresult types; the driver call is reached through the runtime

#include <mutex>

#include "common.cuh"

namespace ttn {
namespace {

constexpr size_t kStaticScratchBytes = (size_t)8 << 20;

// In host code this name is only a host-side stand-in for the device array; the
// kernels must be given the address from cudaGetSymbolAddress.
__device__ __align__(256) unsigned char g_select_scratch[kStaticScratchBytes];

// The calling thread's current context (NULL when none is bound yet), through
// the driver's cuCtxGetCurrent as the runtime exposes it (no libcuda link).
ttn_status current_context(CUcontext* ctx) {
  using GetCurrent = CUresult (*)(CUcontext*);
  static GetCurrent get_current = nullptr;
  static std::once_flag once;
  static cudaError_t lookup = cudaSuccess;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult found = cudaDriverEntryPointSymbolNotFound;
    lookup = cudaGetDriverEntryPoint("cuCtxGetCurrent", (void**)&get_current, cudaEnableDefault, &found);
    if (lookup == cudaSuccess && found != cudaDriverEntryPointSuccess) lookup = cudaErrorNotSupported;
  });
  TTN_TRY(cuda_check(lookup, "ttn_select_f16_static: cuCtxGetCurrent entry point"));
  if (get_current(ctx) != CUDA_SUCCESS)
    return fail(TTN_CUDA_ERROR, "ttn_select_f16_static: cuCtxGetCurrent failed");
  return TTN_OK;
}

ttn_status scratch_address(cudaStream_t stream, void** out) {
  static std::mutex mutex;
  static CUcontext contexts[64] = {nullptr};
  static void* addresses[64] = {nullptr};
  static int used = 0;
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  TTN_TRY(cuda_check(cudaStreamIsCapturing(stream, &capture), "ttn_select_f16_static: cudaStreamIsCapturing"));
  CUcontext ctx = nullptr;
  TTN_TRY(current_context(&ctx));
  std::lock_guard<std::mutex> lock(mutex);
  int slot = -1;
  for (int i = 0; i < used; ++i)
    if (ctx && contexts[i] == ctx) slot = i;
  if (capture != cudaStreamCaptureStatusNone) {
    if (slot < 0)
      return fail(TTN_INVALID_ARG,
                  "ttn_select_f16_static: first call in this CUDA context made during stream capture; "
                  "make one call outside capture first (it resolves the scratch address)");
    *out = addresses[slot];
    return TTN_OK;
  }
  void* p = nullptr;
  TTN_TRY(cuda_check(cudaGetSymbolAddress(&p, g_select_scratch), "ttn_select_f16_static: cudaGetSymbolAddress"));
  if (!ctx) TTN_TRY(current_context(&ctx));  // the lookup bound the device's primary context
  if (slot < 0) {
    for (int i = 0; i < used; ++i)
      if (contexts[i] == ctx) slot = i;
  }
  if (slot < 0) {
    slot = used < 64 ? used++ : 63;  // beyond 64 contexts the last entry is reused
    contexts[slot] = ctx;
  }
  addresses[slot] = p;
  *out = p;
  return TTN_OK;
}

}  // namespace
}  // namespace ttn

using namespace ttn;

extern "C" ttn_status ttn_select_f16_static(const ttn_tensor* decoded, int64_t max_det,
                                            uint32_t flags, float* out,
                                            const ttn_select_trace* trace, ttn_stream stream) {
  const char* name = "ttn_select_f16_static";
  TTN_TRY(validate(decoded, name));
  if (decoded->dtype != TTN_F16 || decoded->ndim != 3)
    return fail(TTN_INVALID_ARG, "%s: detection_select expects FP16 [B,A,4+nc]", name);
  if (decoded->sizes[2] <= 4 || max_det < 0)
    return fail(TTN_INVALID_ARG, "%s: detection_select requires nc > 0 and max_det >= 0", name);
  const size_t need = ttn_select_workspace_size(decoded->sizes[0], decoded->sizes[1],
                                                decoded->sizes[2] - 4, max_det, flags);
  if (need > kStaticScratchBytes)
    return fail(TTN_UNSUPPORTED,
                "%s: this batch needs %zu bytes of scratch; the static scratch holds %zu bytes "
                "(split the batch, or call ttn_select_f16 with your own workspace)",
                name, need, kStaticScratchBytes);
  void* scratch = nullptr;
  TTN_TRY(scratch_address((cudaStream_t)stream, &scratch));
  return ttn_select_f16(decoded, max_det, flags, scratch, kStaticScratchBytes, out, trace, stream);
}
