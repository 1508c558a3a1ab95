// Data movement: strided copy (materialise a view), concat, and the
// NC1HWC0 <-> NCHW layout conversions.  Pure bit movement, so results are
// bit-exact by construction (NaN payloads included).
//
// concat: every input whose rows are dense is one "2-D copy" (outer rows of
// `run` elements at a source pitch into the output at a column offset).  All
// inputs of one call share a single launch: blocks walk a flattened list of
// (input, row, chunk) work items, copying 16-byte vectors when the row start
// addresses allow and scalars otherwise.  Short rows (narrow last-dim cats)
// use one thread per output element instead.  Inputs that are not dense in
// their inner dims are materialised into the output slice by the strided copy.
#include "common.cuh"

namespace ttn {
namespace {

constexpr int kThreads = 256;

// ------------------------------------------------------------- strided copy

template <typename T>
__global__ void __launch_bounds__(kThreads) copy_strided(const T* src, T* dst, Index6 ix, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t os, od, unused;
    offsets3(ix, i, os, od, unused);
    dst[od] = src[os];
  }
}

__global__ void __launch_bounds__(kThreads) copy_dense16(const uint4* src, uint4* dst, int64_t nvec,
                                                         const uint8_t* st, uint8_t* dt, int tail) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + stride < nvec; i += 2 * stride) {
    uint4 a = src[i], b = src[i + stride];
    dst[i] = a;
    dst[i + stride] = b;
  }
  if (i < nvec) dst[i] = src[i];
  if (blockIdx.x == 0 && (int)threadIdx.x < tail) dt[threadIdx.x] = st[threadIdx.x];
}

// Batched 2-D transpose: dst[b][r][c] = src[b][c][r] style copies where the
// destination is contiguous along dim 0 and the source along dim 1.
template <typename T>
__global__ void __launch_bounds__(256) transpose_tiles(const T* src, T* dst, int64_t d0, int64_t d1,
                                                       int64_t batches, int64_t s0, int64_t s1,
                                                       int64_t sb, int64_t t0, int64_t t1,
                                                       int64_t tb) {
  __shared__ T tile[32][33];
  int64_t tiles0 = (d0 + 31) / 32, tiles1 = (d1 + 31) / 32;
  for (int64_t job = blockIdx.x; job < batches * tiles0 * tiles1; job += gridDim.x) {
    int64_t b = job / (tiles0 * tiles1);
    int64_t rem = job % (tiles0 * tiles1);
    int64_t base1 = (rem / tiles0) * 32, base0 = (rem % tiles0) * 32;
    // read: consecutive threads walk dim 1 (source-contiguous)
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
      int64_t i0 = base0 + k, i1 = base1 + threadIdx.x;
      if (i0 < d0 && i1 < d1) tile[k][threadIdx.x] = src[b * sb + i0 * s0 + i1 * s1];
    }
    __syncthreads();
    // write: consecutive threads walk dim 0 (destination-contiguous)
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
      int64_t i1 = base1 + k, i0 = base0 + threadIdx.x;
      if (i0 < d0 && i1 < d1) dst[b * tb + i0 * t0 + i1 * t1] = tile[threadIdx.x][k];
    }
    __syncthreads();
  }
}

// --------------------------------------------------------------- concat

constexpr int kMaxCat = 64;
constexpr int64_t kChunk = 4096;  // elements per work item

struct CatInput {
  const uint8_t* src;
  int64_t src_pitch;   // bytes between rows
  int64_t run;         // bytes per row
  int64_t dst_offset;  // byte column offset in the output row
  int64_t first_item;  // prefix of work items
  int64_t chunks;      // work items per row
};

struct CatPlan {
  int count;
  int64_t outer;
  int64_t dst_pitch;  // bytes
  int64_t items;
  int64_t chunk_bytes;
  uint8_t* dst;
  CatInput in[kMaxCat];
};

__global__ void __launch_bounds__(kThreads) cat_rows(const __grid_constant__ CatPlan plan) {
  for (int64_t item = blockIdx.x; item < plan.items; item += gridDim.x) {
    int lo = 0, hi = plan.count - 1;
    while (lo < hi) {  // last input whose first_item <= item
      int mid = (lo + hi + 1) >> 1;
      if (plan.in[mid].first_item <= item) lo = mid;
      else hi = mid - 1;
    }
    const CatInput& in = plan.in[lo];
    int64_t local = item - in.first_item;
    int64_t row = local / in.chunks, chunk = local % in.chunks;
    int64_t begin = chunk * plan.chunk_bytes;
    int64_t bytes = in.run - begin < plan.chunk_bytes ? in.run - begin : plan.chunk_bytes;
    const uint8_t* s = in.src + row * in.src_pitch + begin;
    uint8_t* d = plan.dst + row * plan.dst_pitch + in.dst_offset + begin;
    if ((((uintptr_t)s | (uintptr_t)d) & 15u) == 0) {
      int64_t nvec = bytes >> 4;
      const uint4* sv = reinterpret_cast<const uint4*>(s);
      uint4* dv = reinterpret_cast<uint4*>(d);
      for (int64_t v = threadIdx.x; v < nvec; v += blockDim.x) dv[v] = sv[v];
      for (int64_t b = nvec * 16 + threadIdx.x; b < bytes; b += blockDim.x) d[b] = s[b];
    } else if ((((uintptr_t)s | (uintptr_t)d | (uintptr_t)bytes) & 1u) == 0) {
      const uint16_t* sh = reinterpret_cast<const uint16_t*>(s);
      uint16_t* dh = reinterpret_cast<uint16_t*>(d);
      for (int64_t v = threadIdx.x; v < bytes / 2; v += blockDim.x) dh[v] = sh[v];
    } else {
      for (int64_t b = threadIdx.x; b < bytes; b += blockDim.x) d[b] = s[b];
    }
  }
}

// Narrow rows: one thread per output element of the concatenated width.
template <typename T>
__global__ void __launch_bounds__(kThreads) cat_elements(const __grid_constant__ CatPlan plan,
                                                         int64_t width) {
  const int64_t total = plan.outer * width;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    int64_t row = i / width, col = i % width;
    int64_t col_bytes = col * (int64_t)sizeof(T);
    int lo = 0, hi = plan.count - 1;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (plan.in[mid].dst_offset <= col_bytes) lo = mid;
      else hi = mid - 1;
    }
    const CatInput& in = plan.in[lo];
    const T* s = reinterpret_cast<const T*>(in.src + row * in.src_pitch + (col_bytes - in.dst_offset));
    T* d = reinterpret_cast<T*>(plan.dst + row * plan.dst_pitch + col_bytes);
    *d = *s;
  }
}

// ------------------------------------------------------------- host side

ttn_status to_index6(const Coalesced& c, Index6& ix, const char* what) {
  if (c.ndim > 6)
    return fail(TTN_UNSUPPORTED, "%s: view needs %d dims after coalescing (max 6)", what, c.ndim);
  ix.ndim = c.ndim;
  for (int d = 0; d < 6; ++d) {
    ix.size[d] = d < c.ndim ? c.size[d] : 1;
    for (int v = 0; v < 3; ++v) ix.stride[v][d] = (d < c.ndim && v < 2) ? c.stride[v][d] : 0;
  }
  return TTN_OK;
}

ttn_status copy_views(const ttn_tensor* src, const ttn_tensor* dst, cudaStream_t s) {
  const ttn_tensor* views[2] = {src, dst};
  Coalesced c = coalesce(views, 2);
  if (!c.numel) return TTN_OK;
  size_t es = dtype_size(src->dtype);
  if (c.ndim == 0 || (c.ndim == 1 && c.stride[0][0] == 1 && c.stride[1][0] == 1)) {
    int64_t bytes = c.numel * (int64_t)es;
    if ((((uintptr_t)src->data | (uintptr_t)dst->data) & 15u) == 0) {
      int64_t nvec = bytes / 16;
      int tail = (int)(bytes - nvec * 16);
      copy_dense16<<<grid_for(nvec ? nvec : 1, kThreads * 2), kThreads, 0, s>>>(
          (const uint4*)src->data, (uint4*)dst->data, nvec,
          (const uint8_t*)src->data + nvec * 16, (uint8_t*)dst->data + nvec * 16, tail);
      return launch_check("ttn_copy");
    }
  }
  // Batched transpose: dst contiguous along coalesced dim 0, src along dim 1.
  if ((c.ndim == 2 || c.ndim == 3) && c.stride[1][0] == 1 && c.stride[0][1] == 1 &&
      c.size[0] >= 8 && c.size[1] >= 8) {
    int64_t batches = c.ndim == 3 ? c.size[2] : 1;
    int64_t sb = c.ndim == 3 ? c.stride[0][2] : 0, tb = c.ndim == 3 ? c.stride[1][2] : 0;
    int64_t jobs = batches * ((c.size[0] + 31) / 32) * ((c.size[1] + 31) / 32);
    unsigned grid = (unsigned)(jobs < (int64_t)sm_count() * 16 ? jobs : (int64_t)sm_count() * 16);
    dim3 block(32, 8);
    if (es == 2)
      transpose_tiles<uint16_t><<<grid, block, 0, s>>>(
          (const uint16_t*)src->data, (uint16_t*)dst->data, c.size[0], c.size[1], batches,
          c.stride[0][0], c.stride[0][1], sb, c.stride[1][0], c.stride[1][1], tb);
    else
      transpose_tiles<uint32_t><<<grid, block, 0, s>>>(
          (const uint32_t*)src->data, (uint32_t*)dst->data, c.size[0], c.size[1], batches,
          c.stride[0][0], c.stride[0][1], sb, c.stride[1][0], c.stride[1][1], tb);
    return launch_check("ttn_copy transpose");
  }
  Index6 ix;
  TTN_TRY(to_index6(c, ix, "ttn_copy"));
  unsigned grid = grid_for(c.numel, kThreads);
  if (es == 2)
    copy_strided<uint16_t><<<grid, kThreads, 0, s>>>((const uint16_t*)src->data,
                                                      (uint16_t*)dst->data, ix, c.numel);
  else
    copy_strided<uint32_t><<<grid, kThreads, 0, s>>>((const uint32_t*)src->data,
                                                      (uint32_t*)dst->data, ix, c.numel);
  return launch_check("ttn_copy");
}

// Row description of a view split at `dim`: rows over dims < dim (must share
// one pitch), dense `run` elements over dims >= dim.  Returns false otherwise.
bool rows_of(const ttn_tensor* t, int dim, int64_t& outer, int64_t& pitch, int64_t& run) {
  int64_t expect = 1;
  run = 1;
  for (int d = t->ndim - 1; d >= dim; --d) {
    if (t->sizes[d] != 1 && t->strides[d] != expect) return false;
    expect *= t->sizes[d];
    run *= t->sizes[d];
  }
  outer = 1;
  pitch = run;
  bool first = true;
  int64_t prev_stride = 0, prev_size = 0;
  for (int d = dim - 1; d >= 0; --d) {
    outer *= t->sizes[d];
    if (t->sizes[d] == 1) continue;
    if (first) {
      pitch = t->strides[d];
      first = false;
    } else if (t->strides[d] != prev_stride * prev_size) {
      return false;
    }
    prev_stride = t->strides[d];
    prev_size = t->sizes[d];
  }
  return true;
}

}  // namespace
}  // namespace ttn

using namespace ttn;

extern "C" {

ttn_status ttn_copy(const ttn_tensor* src, const ttn_tensor* dst, ttn_stream stream) {
  TTN_TRY(validate(src, "ttn_copy src"));
  TTN_TRY(validate(dst, "ttn_copy dst"));
  if (!same_sizes(src, dst)) return fail(TTN_INVALID_ARG, "ttn_copy: sizes differ");
  if (src->dtype != dst->dtype) return fail(TTN_INVALID_ARG, "ttn_copy: dtypes differ");
  return copy_views(src, dst, (cudaStream_t)stream);
}

ttn_status ttn_cat(int32_t count, const ttn_tensor* inputs, int32_t dim, const ttn_tensor* out,
                   ttn_stream stream) {
  const char* name = "ttn_cat";
  if (count <= 0 || !inputs) return fail(TTN_INVALID_ARG, "%s: expects a nonempty tensor list", name);
  TTN_TRY(validate(out, name));
  if (dim < 0 || dim >= out->ndim) return fail(TTN_INVALID_ARG, "%s: dim %d out of range", name, dim);
  int64_t total = 0;
  for (int i = 0; i < count; ++i) {
    const ttn_tensor* t = &inputs[i];
    TTN_TRY(validate(t, name));
    if (!numel(t)) continue;
    if (t->dtype != out->dtype) return fail(TTN_INVALID_ARG, "%s: dtype mismatch", name);
    if (t->ndim != out->ndim) return fail(TTN_INVALID_ARG, "%s: rank mismatch", name);
    for (int d = 0; d < t->ndim; ++d)
      if (d != dim && t->sizes[d] != out->sizes[d])
        return fail(TTN_INVALID_ARG, "%s: shape mismatch outside the concatenation dim", name);
    total += t->sizes[dim];
  }
  if (total != out->sizes[dim])
    return fail(TTN_INVALID_ARG, "%s: output size %lld along dim != sum of inputs %lld", name,
                (long long)out->sizes[dim], (long long)total);
  if (!numel(out)) return TTN_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t es = dtype_size(out->dtype);

  int64_t out_outer, out_pitch, out_run;
  bool out_rows = rows_of(out, dim, out_outer, out_pitch, out_run);
  int64_t inner = 1;
  for (int d = dim + 1; d < out->ndim; ++d) inner *= out->sizes[d];

  CatPlan plan;
  plan.count = 0;
  plan.outer = out_outer;
  plan.dst_pitch = out_pitch * (int64_t)es;
  plan.dst = (uint8_t*)out->data;
  plan.chunk_bytes = kChunk * (int64_t)es;
  plan.items = 0;
  int64_t start = 0;  // along dim
  int64_t runs_total = 0;
  bool pending_fallback = false;
  auto flush = [&]() -> ttn_status {
    if (!plan.count) return TTN_OK;
    int64_t width_bytes = 0;
    for (int i = 0; i < plan.count; ++i) width_bytes += plan.in[i].run;
    int64_t avg_run = width_bytes / plan.count;
    bool contiguous_cover = true;  // inputs tile the whole output row
    int64_t expect = 0;
    for (int i = 0; i < plan.count; ++i) {
      if (plan.in[i].dst_offset != expect) contiguous_cover = false;
      expect += plan.in[i].run;
    }
    if (expect != out_run * (int64_t)es) contiguous_cover = false;
    if (avg_run < 512 && contiguous_cover) {
      int64_t width = out_run;
      unsigned grid = grid_for(plan.outer * width, kThreads);
      if (es == 2) cat_elements<uint16_t><<<grid, kThreads, 0, s>>>(plan, width);
      else cat_elements<uint32_t><<<grid, kThreads, 0, s>>>(plan, width);
    } else {
      unsigned grid = grid_for(plan.items, 1, 16);
      cat_rows<<<grid, kThreads, 0, s>>>(plan);
    }
    plan.count = 0;
    plan.items = 0;
    return launch_check(name);
  };
  // One launch covers up to kMaxCat dense inputs; collect them first.
  struct Pending { int index; int64_t start; };
  Pending fallback[1024];
  int fallback_count = 0;
  for (int i = 0; i < count; ++i) {
    const ttn_tensor* t = &inputs[i];
    int64_t n = numel(t);
    if (!n) continue;
    int64_t outer, pitch, run;
    if (out_rows && rows_of(t, dim, outer, pitch, run) && outer == out_outer) {
      CatInput& e = plan.in[plan.count];
      e.src = (const uint8_t*)t->data;
      e.src_pitch = pitch * (int64_t)es;
      e.run = run * (int64_t)es;
      e.dst_offset = start * inner * (int64_t)es;
      e.chunks = (e.run + plan.chunk_bytes - 1) / plan.chunk_bytes;
      e.first_item = plan.items;
      plan.items += outer * e.chunks;
      runs_total += e.run;
      ++plan.count;
      if (plan.count == kMaxCat) TTN_TRY(flush());
    } else {
      if (fallback_count == 1024) return fail(TTN_UNSUPPORTED, "%s: too many strided inputs", name);
      fallback[fallback_count++] = Pending{i, start};
      pending_fallback = true;
    }
    start += t->sizes[dim];
  }
  TTN_TRY(flush());
  if (pending_fallback) {
    for (int f = 0; f < fallback_count; ++f) {
      const ttn_tensor* t = &inputs[fallback[f].index];
      ttn_tensor slice = *out;
      slice.sizes[dim] = t->sizes[dim];
      slice.data = (uint8_t*)out->data + fallback[f].start * out->strides[dim] * (int64_t)es;
      TTN_TRY(copy_views(t, &slice, s));
    }
  }
  (void)runs_total;
  return TTN_OK;
}

}  // extern "C"
