// Runtime half of libttn: status strings, the per-thread error message, view
// validation/coalescing shared by every op, and the C-side stream-capture
// graph (the CUDA twin of the reference's RuntimeGraph, backend.cpp:62-113).
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <tuple>
#include <mutex>
#include <thread>

#include "common.cuh"

namespace ttn {

static thread_local char g_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, args);
  va_end(args);
}

ttn_status fail(ttn_status status, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, args);
  va_end(args);
  return status;
}

int sm_count() {
  static std::mutex mutex;
  static int cached[64] = {0};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 148;
  std::lock_guard<std::mutex> lock(mutex);
  if (!cached[device]) {
    int count = 0;
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        count <= 0)
      count = 148;
    cached[device] = count;
  }
  return cached[device];
}

ttn_status ensure_dynamic_smem(const void* kernel, int bytes) {
  static std::mutex mutex;
  static std::map<std::pair<int, const void*>, int> granted;  // dynamic bytes a launch may use
  if (bytes <= 0) return TTN_OK;
  int device = 0;
  TTN_TRY(cuda_check(cudaGetDevice(&device), "cudaGetDevice"));
  std::lock_guard<std::mutex> lock(mutex);
  auto key = std::make_pair(device, kernel);
  auto it = granted.find(key);
  if (it == granted.end()) {  // the default: 48 KB less the kernel's static shared memory
    cudaFuncAttributes attr;
    TTN_TRY(cuda_check(cudaFuncGetAttributes(&attr, kernel), "cudaFuncGetAttributes"));
    it = granted.emplace(key, attr.maxDynamicSharedSizeBytes).first;
  }
  if (it->second >= bytes) return TTN_OK;
  TTN_TRY(cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                     "cudaFuncSetAttribute"));
  it->second = bytes;
  return TTN_OK;
}

int resident_blocks(const void* kernel, int threads, size_t smem) {
  static std::mutex mutex;
  static std::map<std::tuple<int, const void*, int, size_t>, int> cache;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return 1;
  std::lock_guard<std::mutex> lock(mutex);
  auto key = std::make_tuple(device, kernel, threads, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, threads, smem) != cudaSuccess ||
      blocks < 1)
    blocks = 1;
  cache[key] = blocks;
  return blocks;
}

namespace {
struct Branch {
  cudaStream_t aux = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
thread_local Branch t_branch[64];  // per host thread and device: calls on one thread are ordered
}  // namespace

ttn_status branch_fork(cudaStream_t stream, cudaStream_t* aux) {
  int device = 0;
  TTN_TRY(cuda_check(cudaGetDevice(&device), "cudaGetDevice"));
  if (device < 0 || device >= 64) return fail(TTN_UNSUPPORTED, "branch_fork: device %d", device);
  Branch& b = t_branch[device];
  if (!b.aux) {
    TTN_TRY(cuda_check(cudaStreamCreateWithFlags(&b.aux, cudaStreamNonBlocking), "cudaStreamCreate"));
    TTN_TRY(cuda_check(cudaEventCreateWithFlags(&b.fork, cudaEventDisableTiming), "cudaEventCreate"));
    TTN_TRY(cuda_check(cudaEventCreateWithFlags(&b.join, cudaEventDisableTiming), "cudaEventCreate"));
  }
  TTN_TRY(cuda_check(cudaEventRecord(b.fork, stream), "cudaEventRecord"));
  TTN_TRY(cuda_check(cudaStreamWaitEvent(b.aux, b.fork, 0), "cudaStreamWaitEvent"));
  *aux = b.aux;
  return TTN_OK;
}

ttn_status branch_join(cudaStream_t stream) {
  int device = 0;
  TTN_TRY(cuda_check(cudaGetDevice(&device), "cudaGetDevice"));
  Branch& b = t_branch[device];
  TTN_TRY(cuda_check(cudaEventRecord(b.join, b.aux), "cudaEventRecord"));
  return cuda_check(cudaStreamWaitEvent(stream, b.join, 0), "cudaStreamWaitEvent");
}

int max_dynamic_smem() {
  static std::mutex mutex;
  static int cached[64] = {0};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 48 * 1024;
  std::lock_guard<std::mutex> lock(mutex);
  if (!cached[device]) {
    int value = 0;
    if (cudaDeviceGetAttribute(&value, cudaDevAttrMaxSharedMemoryPerBlockOptin, device) != cudaSuccess ||
        value <= 0)
      value = 48 * 1024;
    cached[device] = value;
  }
  return cached[device];
}

ttn_status validate(const ttn_tensor* t, const char* name) {
  if (!t) return fail(TTN_INVALID_ARG, "%s: null descriptor", name);
  if (t->ndim < 0 || t->ndim > TTN_MAX_DIMS)
    return fail(TTN_INVALID_ARG, "%s: ndim %d outside [0, %d]", name, t->ndim, TTN_MAX_DIMS);
  if (t->dtype != TTN_F16 && t->dtype != TTN_F32)
    return fail(TTN_UNSUPPORTED, "%s: dtype %d is not float16/float32", name, t->dtype);
  int64_t count = 1;
  for (int d = 0; d < t->ndim; ++d) {
    if (t->sizes[d] < 0) return fail(TTN_INVALID_ARG, "%s: negative size", name);
    count *= t->sizes[d];
  }
  if (count && !t->data) return fail(TTN_INVALID_ARG, "%s: null data pointer", name);
  uintptr_t addr = (uintptr_t)t->data;
  if (count && addr % dtype_size(t->dtype))
    return fail(TTN_INVALID_ARG, "%s: data pointer not aligned to its element size", name);
  return TTN_OK;
}

bool same_sizes(const ttn_tensor* a, const ttn_tensor* b) {
  if (a->ndim != b->ndim) return false;
  for (int d = 0; d < a->ndim; ++d)
    if (a->sizes[d] != b->sizes[d]) return false;
  return true;
}

int64_t numel(const ttn_tensor* t) {
  int64_t count = 1;
  for (int d = 0; d < t->ndim; ++d) count *= t->sizes[d];
  return count;
}

bool is_contiguous(const ttn_tensor* t) {
  int64_t expect = 1;
  for (int d = t->ndim - 1; d >= 0; --d) {
    if (t->sizes[d] == 1) continue;
    if (t->strides[d] != expect) return false;
    expect *= t->sizes[d];
  }
  return true;
}

Coalesced coalesce(const ttn_tensor* const* views, int count) {
  Coalesced c;
  const ttn_tensor* first = views[0];
  for (int d = first->ndim - 1; d >= 0; --d) {
    int64_t size = first->sizes[d];
    c.numel *= size;
    if (size == 1) continue;
    bool merge = c.ndim > 0;
    for (int v = 0; v < count && merge; ++v)
      if (c.stride[v][c.ndim - 1] * c.size[c.ndim - 1] != views[v]->strides[d]) merge = false;
    if (merge) {
      c.size[c.ndim - 1] *= size;
    } else {
      c.size[c.ndim] = size;
      for (int v = 0; v < count; ++v) c.stride[v][c.ndim] = views[v]->strides[d];
      ++c.ndim;
    }
  }
  if (first->ndim == 0) c.numel = 1;
  return c;
}

}  // namespace ttn

using namespace ttn;

struct ttn_graph {
  cudaStream_t stream = nullptr;
  cudaGraphExec_t exec = nullptr;
  std::thread::id owner = std::this_thread::get_id();
  bool active = false;
  bool closed = false;
};

extern "C" {

int ttn_version(void) { return 100; }

const char* ttn_status_string(ttn_status status) {
  switch (status) {
    case TTN_OK: return "TTN_OK";
    case TTN_INVALID_ARG: return "TTN_INVALID_ARG";
    case TTN_UNSUPPORTED: return "TTN_UNSUPPORTED";
    case TTN_CUDA_ERROR: return "TTN_CUDA_ERROR";
    case TTN_TIMEOUT: return "TTN_TIMEOUT";
    case TTN_DEVICE_FAULT_FLAG: return "TTN_DEVICE_FAULT_FLAG";
  }
  return "TTN_UNKNOWN_STATUS";
}

const char* ttn_last_error(void) { return g_error; }

static size_t round_blocks(size_t bytes) { return (bytes + 31) / 32 * 32; }

ttn_status ttn_malloc(void** ptr, size_t bytes) {
  if (!ptr) return fail(TTN_INVALID_ARG, "ttn_malloc: null output");
  *ptr = nullptr;
  if (!bytes) return TTN_OK;
  if (bytes > SIZE_MAX - 31) return fail(TTN_INVALID_ARG, "ttn_malloc: size overflows");
  return cuda_check(cudaMalloc(ptr, round_blocks(bytes)), "ttn_malloc");
}

ttn_status ttn_free(void* ptr) { return ptr ? cuda_check(cudaFree(ptr), "ttn_free") : TTN_OK; }

ttn_status ttn_malloc_host(void** ptr, size_t bytes) {
  if (!ptr) return fail(TTN_INVALID_ARG, "ttn_malloc_host: null output");
  *ptr = nullptr;
  if (!bytes) return TTN_OK;
  if (bytes > SIZE_MAX - 31) return fail(TTN_INVALID_ARG, "ttn_malloc_host: size overflows");
  return cuda_check(cudaMallocHost(ptr, round_blocks(bytes)), "ttn_malloc_host");
}

ttn_status ttn_free_host(void* ptr) { return ptr ? cuda_check(cudaFreeHost(ptr), "ttn_free_host") : TTN_OK; }

ttn_status ttn_memcpy_async(void* dst, const void* src, size_t bytes, int kind, ttn_stream stream) {
  static const cudaMemcpyKind kinds[3] = {cudaMemcpyHostToDevice, cudaMemcpyDeviceToHost,
                                          cudaMemcpyDeviceToDevice};
  if (kind < 0 || kind > 2) return fail(TTN_INVALID_ARG, "ttn_memcpy_async: unknown kind %d", kind);
  if (!bytes) return TTN_OK;
  if (!dst || !src) return fail(TTN_INVALID_ARG, "ttn_memcpy_async: null pointer");
  return cuda_check(cudaMemcpyAsync(dst, src, bytes, kinds[kind], (cudaStream_t)stream), "ttn_memcpy_async");
}

ttn_status ttn_graph_create(ttn_graph** graph) {
  if (!graph) return fail(TTN_INVALID_ARG, "ttn_graph_create: null output");
  *graph = new (std::nothrow) ttn_graph();
  return *graph ? TTN_OK : fail(TTN_INVALID_ARG, "ttn_graph_create: out of host memory");
}

static ttn_status same_thread(const ttn_graph* g, const char* what) {
  if (!g) return fail(TTN_INVALID_ARG, "%s: null graph", what);
  if (g->owner != std::this_thread::get_id())
    return fail(TTN_INVALID_ARG, "%s: RuntimeGraph must stay on its creating thread/stream", what);
  return TTN_OK;
}

ttn_status ttn_graph_begin(ttn_graph* g, ttn_stream stream) {
  TTN_TRY(same_thread(g, "ttn_graph_begin"));
  if (g->closed || g->active || g->exec)
    return fail(TTN_INVALID_ARG, "RuntimeGraph cannot begin in its current state");
  cudaStream_t s = (cudaStream_t)stream;
  if (!s) return fail(TTN_INVALID_ARG, "ttn_graph_begin: the legacy default stream cannot be captured");
  cudaStreamCaptureStatus status;
  TTN_TRY(cuda_check(cudaStreamIsCapturing(s, &status), "cudaStreamIsCapturing"));
  if (status != cudaStreamCaptureStatusNone)
    return fail(TTN_INVALID_ARG, "ttn_graph_begin: stream is already capturing");
  TTN_TRY(cuda_check(cudaStreamSynchronize(s), "cudaStreamSynchronize"));
  TTN_TRY(cuda_check(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal),
                     "cudaStreamBeginCapture"));
  g->stream = s;
  g->active = true;
  return TTN_OK;
}

ttn_status ttn_graph_end(ttn_graph* g) {
  TTN_TRY(same_thread(g, "ttn_graph_end"));
  if (!g->active) return fail(TTN_INVALID_ARG, "RuntimeGraph is not capturing");
  cudaGraph_t graph = nullptr;
  cudaError_t err = cudaStreamEndCapture(g->stream, &graph);
  g->active = false;
  TTN_TRY(cuda_check(err, "cudaStreamEndCapture"));
  err = cudaGraphInstantiate(&g->exec, graph, 0);
  cudaGraphDestroy(graph);
  return cuda_check(err, "cudaGraphInstantiate");
}

ttn_status ttn_graph_replay(ttn_graph* g) {
  TTN_TRY(same_thread(g, "ttn_graph_replay"));
  if (g->closed || !g->exec || g->active)
    return fail(TTN_INVALID_ARG, "RuntimeGraph is not ready to replay");
  return cuda_check(cudaGraphLaunch(g->exec, g->stream), "cudaGraphLaunch");
}

ttn_status ttn_graph_close(ttn_graph* g) {
  TTN_TRY(same_thread(g, "ttn_graph_close"));
  if (g->closed) return TTN_OK;
  if (g->active) TTN_TRY(ttn_graph_end(g));
  if (g->exec) {
    TTN_TRY(cuda_check(cudaStreamSynchronize(g->stream), "cudaStreamSynchronize"));
    TTN_TRY(cuda_check(cudaGraphExecDestroy(g->exec), "cudaGraphExecDestroy"));
    g->exec = nullptr;
  }
  g->closed = true;
  return TTN_OK;
}

void ttn_graph_destroy(ttn_graph* g) {
  if (!g) return;
  if (g->owner == std::this_thread::get_id()) ttn_graph_close(g);
  delete g;
}

}  // extern "C"
