// fp16 SiLU and sigmoid as 65,536-entry tables, one value per input bit
// pattern, built on the device by the exact routines (silu_h / sigmoid_h, the
// PyTorch CPU eager rule) the first time a kernel asks for them.  An fp16 input
// has only 2^16 values, so a table read returns exactly what the exact routine
// returns for that input.
#include <mutex>

#include "common.cuh"

namespace ttn {
namespace {

__device__ __align__(16) uint16_t g_unary_tables[2][65536];  // [kind][input bits]

__global__ void __launch_bounds__(256) build_unary_tables(uint16_t* tables) {
  const uint32_t bits = blockIdx.x * 256u + threadIdx.x;  // grid covers 65,536 exactly
  tables[bits] = silu_h((uint16_t)bits);
  tables[65536 + bits] = sigmoid_h((uint16_t)bits);
}

}  // namespace

ttn_status unary_table(int kind, cudaStream_t stream, const uint16_t** table) {
  static std::mutex mutex;
  static uint16_t* base[64] = {nullptr};
  static bool ready[64] = {false};
  if (kind != 0 && kind != 1) return fail(TTN_INVALID_ARG, "unary_table: kind %d", kind);
  int device = 0;
  TTN_TRY(cuda_check(cudaGetDevice(&device), "cudaGetDevice"));
  if (device < 0 || device >= 64) return fail(TTN_UNSUPPORTED, "unary_table: device %d", device);
  std::lock_guard<std::mutex> lock(mutex);
  if (!base[device]) {
    void* p = nullptr;
    TTN_TRY(cuda_check(cudaGetSymbolAddress(&p, g_unary_tables), "cudaGetSymbolAddress"));
    base[device] = (uint16_t*)p;
  }
  if (!ready[device]) {
    // Built on the caller's stream, so the caller's next kernel sees it.  Under
    // stream capture the build becomes part of the graph (and runs with every
    // replay) until an uncaptured call has built and synchronised it once.
    cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
    TTN_TRY(cuda_check(cudaStreamIsCapturing(stream, &status), "cudaStreamIsCapturing"));
    build_unary_tables<<<256, 256, 0, stream>>>(base[device]);
    TTN_TRY(launch_check("build_unary_tables"));
    if (status == cudaStreamCaptureStatusNone) {
      TTN_TRY(cuda_check(cudaStreamSynchronize(stream), "build_unary_tables"));
      ready[device] = true;
    }
  }
  *table = base[device] + (size_t)kind * 65536;
  return TTN_OK;
}

}  // namespace ttn
