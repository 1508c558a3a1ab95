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
//  * the first call on a device resolves the array's device address with
//    cudaGetSymbolAddress (once per device, with that device current), so make
//    that first call before any stream capture.
// The entry point itself calls no cudaMalloc, cudaFree or other allocating
// routine.
#include <mutex>

#include "common.cuh"

namespace ttn {
namespace {

constexpr size_t kStaticScratchBytes = (size_t)8 << 20;

// In host code this name is only a host-side stand-in for the device array; the
// kernels must be given the address from cudaGetSymbolAddress.
__device__ __align__(256) unsigned char g_select_scratch[kStaticScratchBytes];

ttn_status scratch_address(void** out) {
  static std::mutex mutex;
  static void* address[64] = {nullptr};
  int device = 0;
  TTN_TRY(cuda_check(cudaGetDevice(&device), "ttn_select_f16_static: cudaGetDevice"));
  if (device < 0 || device >= 64)
    return fail(TTN_UNSUPPORTED, "ttn_select_f16_static: device index %d out of range", device);
  std::lock_guard<std::mutex> lock(mutex);
  if (!address[device]) {
    void* p = nullptr;
    TTN_TRY(cuda_check(cudaGetSymbolAddress(&p, g_select_scratch),
                       "ttn_select_f16_static: cudaGetSymbolAddress"));
    address[device] = p;
  }
  *out = address[device];
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
  TTN_TRY(scratch_address(&scratch));
  return ttn_select_f16(decoded, max_det, flags, scratch, kStaticScratchBytes, out, trace, stream);
}
