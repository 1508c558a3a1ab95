// Elementwise ops of the op pass: SiLU, sigmoid, add/sub/mul/div (tensor or
// scalar operand, stride-0 broadcast) and the fused NC1HWC0 y = SiLU(x+b)+r.
//
// HBM-bound: the contiguous paths move 16 bytes per thread per access (8 fp16
// lanes, 128-bit loads/stores) with two independent accesses in flight per
// thread, on a grid-stride loop sized to a few waves of the 148 SMs.  Views
// that are not dense fall back to one thread per element over a coalesced
// index space (<= 6 dims).  All arithmetic is FP32 with one rounding to fp16,
// the rule of PyTorch CPU eager (and of elementwise.cpp:71-86 in the reference).
#include "common.cuh"

namespace ttn {
namespace {

constexpr int kThreads = 256;

enum UnaryKind { kSilu = 0, kSigmoid = 1 };

template <int K>
__device__ __forceinline__ uint16_t unary_h(uint16_t x) {
  return K == kSilu ? silu_h(x) : sigmoid_h(x);
}
template <int K>
__device__ __forceinline__ float unary_f(float x) {
  return K == kSilu ? silu_f(x) : sigmoid_f(x);
}

template <int K>
__device__ __forceinline__ uint4 unary_vec8(uint4 v) {
  return make_uint4(unary_h2_fast<K == kSilu>(v.x), unary_h2_fast<K == kSilu>(v.y),
                    unary_h2_fast<K == kSilu>(v.z), unary_h2_fast<K == kSilu>(v.w));
}

// Vectorised fp16 SiLU / sigmoid (x may equal y).  Warp-uniform loop: each lane
// owns four 16-byte vectors per step.  A pair whose fast result is not provably
// the CPU's fp16 value (about 1.5% of pairs) is stored with its *input* bits
// unchanged and its element indices go to a per-warp shared-memory queue; when the queue fills
// (and once at the end) the warp re-reads those inputs and writes the exact
// results, 32 elements at a time with every lane busy.  So the exact path costs
// per flagged element rather than per diverged warp step, and works in place.
// Launches cover fewer than 2^32 elements (the host splits larger tensors).
constexpr int kQueue = 256;  // element entries per warp
constexpr int kVec = 4;      // 16-byte vectors per lane per step

// Rewrites the queued elements with the exact routine (yh[e] still holds the
// input bits, stored unchanged).  Each lane gathers four entries before
// computing, so a full queue costs two rounds of L2 latency, not eight.
template <int K>
__device__ __forceinline__ void drain_queue(const uint32_t* queue, int count, uint16_t* yh, int lane) {
  constexpr int kBatch = 4;
  __syncwarp();
  for (int t0 = 0; t0 < count; t0 += 32 * kBatch) {
    uint32_t e[kBatch];
    uint16_t v[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int t = t0 + j * 32 + lane;
      e[j] = t < count ? queue[t] : 0xffffffffu;
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
      if (e[j] != 0xffffffffu) v[j] = yh[e[j]];
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
      if (e[j] != 0xffffffffu) yh[e[j]] = unary_h<K>(v[j]);
  }
  __syncwarp();
}

// Applies the fast core to one lane's kVec vectors in place.  Returns bit
// (4u + w) set where word w of vector u must come from the exact routine; such
// words keep their input bits for the exact pass.
template <int K>
__device__ __forceinline__ uint32_t fast_step(uint4 (&v)[kVec]) {
  uint32_t flags = 0;
#pragma unroll
  for (int u = 0; u < kVec; ++u) {
    uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      bool bad;
      uint32_t r = unary_h2_deferred<K == kSilu>(w[k], bad);
      w[k] = bad ? w[k] : r;
      flags |= bad ? (1u << (4 * u + k)) : 0u;
    }
    v[u] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  return flags;
}

// Queues the flagged pairs of one warp step whose vectors start at vector
// `base` of the row at element offset oy of y (draining the queue first when it
// would overflow; a step with more flagged pairs than the queue holds is
// finished right away).
template <int K>
__device__ __forceinline__ void queue_step(uint32_t flags, int64_t base, int64_t oy, uint16_t* y,
                                           uint32_t* queue, int* q_count, int& count, int lane) {
  if (!__any_sync(0xffffffffu, flags)) return;
  const int mine = 2 * __popc(flags);
  const int total = __reduce_add_sync(0xffffffffu, mine);
  if (count + total > kQueue) {  // make room
    drain_queue<K>(queue, count, y, lane);
    if (lane == 0) *q_count = 0;
    __syncwarp();
    count = 0;
  }
  if (total > kQueue) {  // pathological step: finish its pairs right away
    __syncwarp();
    for (uint32_t f = flags; f; f &= f - 1) {
      int bit = __ffs(f) - 1;
      int64_t e = oy + (base + (bit >> 2) * 32 + lane) * 8 + (bit & 3) * 2;
      y[e] = unary_h<K>(y[e]);
      y[e + 1] = unary_h<K>(y[e + 1]);
    }
    __syncwarp();
    return;
  }
  if (mine) {
    int slot = atomicAdd(q_count, mine);
    for (uint32_t f = flags; f; f &= f - 1) {
      int bit = __ffs(f) - 1;
      uint32_t e = (uint32_t)(oy + (base + (bit >> 2) * 32 + lane) * 8 + (bit & 3) * 2);
      queue[slot] = e;
      queue[slot + 1] = e + 1;
      slot += 2;
    }
  }
  count += total;
}

// rows x vec_per_row 16-byte vectors; row r of x/y starts at the offsets that
// `outer` gives for r.  blockIdx.y walks rows, blockIdx.x / warps walk the
// vectors of a row.  Queue entries are element offsets from y (the host keeps
// y's extent below 2^32 elements).
template <int K>
__global__ void __launch_bounds__(kThreads) unary_f16_vec(const uint16_t* x, uint16_t* y, Index6 outer,
                                                          int64_t vec_per_row, int64_t rows) {
  __shared__ uint32_t queue[kThreads / 32][kQueue];
  __shared__ int q_count[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t step = (int64_t)gridDim.x * (kThreads / 32) * 32 * kVec;
  if (lane == 0) q_count[warp] = 0;
  __syncwarp();
  int count = 0;  // warp-uniform copy of q_count[warp]
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    int64_t ox = 0, oy = 0, unused;
    if (outer.ndim) offsets3(outer, row, ox, oy, unused);
    const uint4* xs = reinterpret_cast<const uint4*>(x + ox);
    uint4* ys = reinterpret_cast<uint4*>(y + oy);
    for (int64_t base = ((int64_t)blockIdx.x * (kThreads / 32) + warp) * 32 * kVec; base < vec_per_row;
         base += step) {
      uint4 v[kVec];
#pragma unroll
      for (int u = 0; u < kVec; ++u) {
        int64_t i = base + u * 32 + lane;
        v[u] = i < vec_per_row ? xs[i] : make_uint4(0, 0, 0, 0);
      }
      uint32_t flags = fast_step<K>(v);
#pragma unroll
      for (int u = 0; u < kVec; ++u) {
        int64_t i = base + u * 32 + lane;
        if (i < vec_per_row) ys[i] = v[u];
        else flags &= ~(0xfu << (4 * u));
      }
      queue_step<K>(flags, base, oy, y, queue[warp], &q_count[warp], count, lane);
    }
  }
  drain_queue<K>(queue[warp], count, y, lane);
}

// Dense fp16, 16-byte aligned, arithmetic core (used below the table path's
// size threshold): nvec 16-byte vectors plus a scalar tail; x may equal y.
// Warp tiles (32 lanes x kVec vectors) go round-robin over all warps of a
// one-wave grid, the next tile prefetched into registers while the current one
// is computed.
constexpr int kTileVecs = 32 * kVec;

template <int K>
__global__ void __launch_bounds__(kThreads) unary_f16_dense(const uint16_t* x, uint16_t* y, int nvec,
                                                               const uint16_t* xt, uint16_t* yt, int tail) {
  __shared__ uint32_t queue[kThreads / 32][kQueue];
  __shared__ int q_count[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint4* xs = reinterpret_cast<const uint4*>(x) + lane;
  uint4* ys = reinterpret_cast<uint4*>(y) + lane;
  const int full = nvec / kTileVecs;
  const int tiles = (nvec + kTileVecs - 1) / kTileVecs;
  const int warps = gridDim.x * (kThreads / 32);
  int tile = blockIdx.x * (kThreads / 32) + warp;
  if (lane == 0) q_count[warp] = 0;
  __syncwarp();
  pdl_trigger();
  pdl_wait();
  int count = 0;
  uint4 next[kVec];
  auto fetch = [&](int t) {
    const uint4* src = xs + (size_t)t * kTileVecs;
    if (t < full) {
#pragma unroll
      for (int u = 0; u < kVec; ++u) next[u] = src[u * 32];
    } else if (t < tiles) {
#pragma unroll
      for (int u = 0; u < kVec; ++u)
        next[u] = t * kTileVecs + u * 32 + lane < nvec ? src[u * 32] : make_uint4(0, 0, 0, 0);
    }
  };
  fetch(tile);
  for (; tile < tiles; tile += warps) {
    uint4 v[kVec];
#pragma unroll
    for (int u = 0; u < kVec; ++u) v[u] = next[u];
    fetch(tile + warps);
    const int base = tile * kTileVecs;
    uint32_t flags = fast_step<K>(v);
    if (tile < full) {
#pragma unroll
      for (int u = 0; u < kVec; ++u) ys[base + u * 32] = v[u];
    } else {
#pragma unroll
      for (int u = 0; u < kVec; ++u) {
        if (base + u * 32 + lane < nvec) ys[base + u * 32] = v[u];
        else flags &= ~(0xfu << (4 * u));
      }
    }
    queue_step<K>(flags, base, 0, y, queue[warp], &q_count[warp], count, lane);
  }
  drain_queue<K>(queue[warp], count, y, lane);
  if (blockIdx.x == 0 && (int)threadIdx.x < tail) yt[threadIdx.x] = unary_h<K>(xt[threadIdx.x]);
}

// Table core for dense fp16 and for two-level row families: one block per SM
// (768 threads) copies the op's 128 KB table into shared memory, then maps
// 16-byte vectors with one shared-memory read per element and no
// transcendental work.  The loads go through a per-thread ring of kLutSlots
// shared-memory slots filled by cp.async, so kLutSlots - 1 vectors per thread
// (48 KB per SM) are always in flight while one is mapped; a thread only reads
// back its own slots, so the ring needs no block barrier.  The table copy is
// the first cp.async group and overlaps the first loads.  Vector g of the
// launch is the thread's (g - first) / stride-th; with kRows its (row, column)
// and the row's (i1, i2) come from multiply-high divisions, else it sits at
// element 8 g.  Fewer than 2^31 vectors per launch; x may equal y.
constexpr int kLutThreads = 768;
constexpr int kLutSlots = 5;
constexpr int kLutBytes = 65536 * 2;
constexpr int kLutSmem = kLutBytes + kLutSlots * kLutThreads * 16;
constexpr int64_t kLutMinVecs = (int64_t)1 << 21;  // below ~17M elements the table copy does not pay

__device__ __forceinline__ uint32_t lut_word(const uint16_t* lut, uint32_t w) {
  return (uint32_t)lut[w & 0xffffu] | ((uint32_t)lut[w >> 16] << 16);
}
__device__ __forceinline__ uint4 lut_vec(const uint16_t* lut, uint4 v) {
  return make_uint4(lut_word(lut, v.x), lut_word(lut, v.y), lut_word(lut, v.z), lut_word(lut, v.w));
}

// Element offsets of x and y for vector g: dense (kRows false) or a row family
// [n1][n2][vpr vectors] with element strides xs1/xs2 and ys1/ys2.
struct LutRows {
  int64_t xs1, xs2, ys1, ys2;
  FastDiv vpr, n2;
};

template <bool kRows>
__device__ __forceinline__ int64_t lut_offset(const LutRows& r, uint32_t g, bool of_y) {
  if constexpr (!kRows) {
    return (int64_t)g * 8;
  } else {
    const uint32_t row = r.vpr.div(g), col = g - row * r.vpr.d;
    const uint32_t i1 = r.n2.div(row), i2 = row - i1 * r.n2.d;
    return of_y ? (int64_t)i1 * r.ys1 + (int64_t)i2 * r.ys2 + (int64_t)col * 8
                : (int64_t)i1 * r.xs1 + (int64_t)i2 * r.xs2 + (int64_t)col * 8;
  }
}

template <bool kRows>
__global__ void __launch_bounds__(kLutThreads, 1) unary_f16_lut(const uint16_t* table, const uint16_t* x,
                                                                uint16_t* y, LutRows rows, uint32_t total,
                                                                const uint16_t* xt, uint16_t* yt, int tail) {
  extern __shared__ __align__(16) uint8_t lut_smem[];
  uint16_t* lut = reinterpret_cast<uint16_t*>(lut_smem);
  uint4* ring = reinterpret_cast<uint4*>(lut_smem + kLutBytes) + threadIdx.x;
  const uint32_t stride = gridDim.x * kLutThreads;  // total < 2^31: g + kLutSlots * stride fits
  const uint32_t first = blockIdx.x * kLutThreads + threadIdx.x;
  {
    const uint4* src = reinterpret_cast<const uint4*>(table);
    uint4* dst = reinterpret_cast<uint4*>(lut);
    for (int t = threadIdx.x; t < kLutBytes / 16; t += kLutThreads) cp_async16(dst + t, src + t);
    cp_async_commit();
  }
  pdl_trigger();  // the table is built once per device, never written by a predecessor
  pdl_wait();
#pragma unroll
  for (int k = 0; k < kLutSlots - 1; ++k) {
    const uint32_t g = first + k * stride;
    if (g < total) cp_async16(ring + k * kLutThreads, x + lut_offset<kRows>(rows, g, false));
    cp_async_commit();
  }
  cp_async_wait<kLutSlots - 1>();  // the table group has landed (for this thread's part)
  __syncthreads();                 // ... and for every thread's part
  int slot = 0;
  for (uint32_t g = first; g < total; g += stride) {
    const uint32_t ahead = g + (kLutSlots - 1) * stride;
    const int refill = slot == 0 ? kLutSlots - 1 : slot - 1;  // the slot mapped last iteration
    if (ahead < total) cp_async16(ring + refill * kLutThreads, x + lut_offset<kRows>(rows, ahead, false));
    cp_async_commit();
    cp_async_wait<kLutSlots - 1>();  // the group that filled `slot`
    const uint4 v = ring[slot * kLutThreads];
    *reinterpret_cast<uint4*>(y + lut_offset<kRows>(rows, g, true)) = lut_vec(lut, v);
    slot = slot == kLutSlots - 1 ? 0 : slot + 1;
  }
  cp_async_wait<0>();
  if (blockIdx.x == 0 && (int)threadIdx.x < tail) yt[threadIdx.x] = lut[xt[threadIdx.x]];
}

// Launches the table kernel over `total` vectors (< 2^31) on the current device.
template <bool kRows>
ttn_status launch_lut(int kind, const uint16_t* x, uint16_t* y, const LutRows& rows, int64_t total,
                      const uint16_t* xt, uint16_t* yt, int tail, cudaStream_t s, const char* name) {
  const uint16_t* table = nullptr;
  TTN_TRY(unary_table(kind, s, &table));
  TTN_TRY(ensure_dynamic_smem((const void*)unary_f16_lut<kRows>, kLutSmem));
  const int64_t want = (total + 4 * kLutThreads - 1) / (4 * kLutThreads);
  const unsigned grid = (unsigned)(want < sm_count() ? (want < 1 ? 1 : want) : sm_count());
  TTN_TRY(cuda_check(launch_pdl(unary_f16_lut<kRows>, grid, kLutThreads, kLutSmem, s, table, x, y, rows,
                                (uint32_t)total, xt, yt, tail),
                     name));
  return launch_check(name);
}

// y = a + SiLU(raw), the residual add of a bottleneck whose second operand is a
// conv output that nothing else reads: the SiLU table kernel with a second input.
// Per element SiLU(raw) comes from the table (the exact fp16 value), then the add
// runs as the binary kernels do, in FP32 with one rounding to fp16 -- bit-identical
// to SiLU followed by the add.  raw and a stream through a per-thread ring of
// kAddSlots slot pairs (2 x 16 bytes each), beside the 128 KB table.  Rows: n1 rows
// of vpr vectors, element strides rs (raw), as (a) and ys (y) between rows.
constexpr int kAddSlots = 4;
constexpr int kAddSmem = kLutBytes + kAddSlots * kLutThreads * 32;

struct AddRows {
  int64_t rs, as, ys;
  FastDiv vpr;
};

__device__ __forceinline__ uint32_t add_word(uint32_t a, uint32_t b) {
  const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&a));
  const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&b));
  const __half2 h = __floats2half2_rn(__fadd_rn(fa.x, fb.x), __fadd_rn(fa.y, fb.y));
  return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void __launch_bounds__(kLutThreads, 1) add_silu_lut(const uint16_t* table, const uint16_t* raw,
                                                               const uint16_t* a, uint16_t* y, AddRows rows,
                                                               uint32_t total) {
  extern __shared__ __align__(16) uint8_t lut_smem[];
  uint16_t* lut = reinterpret_cast<uint16_t*>(lut_smem);
  uint4* ring_r = reinterpret_cast<uint4*>(lut_smem + kLutBytes) + threadIdx.x;
  uint4* ring_a = ring_r + kAddSlots * kLutThreads;
  const uint32_t stride = gridDim.x * kLutThreads;
  const uint32_t first = blockIdx.x * kLutThreads + threadIdx.x;
  auto fetch = [&](int slot, uint32_t g) {
    const uint32_t row = rows.vpr.div(g), col = g - row * rows.vpr.d;
    cp_async16(ring_r + slot * kLutThreads, raw + (int64_t)row * rows.rs + (int64_t)col * 8);
    cp_async16(ring_a + slot * kLutThreads, a + (int64_t)row * rows.as + (int64_t)col * 8);
  };
  {
    const uint4* src = reinterpret_cast<const uint4*>(table);
    uint4* dst = reinterpret_cast<uint4*>(lut);
    for (int t = threadIdx.x; t < kLutBytes / 16; t += kLutThreads) cp_async16(dst + t, src + t);
    cp_async_commit();
  }
  pdl_trigger();
  pdl_wait();
#pragma unroll
  for (int k = 0; k < kAddSlots - 1; ++k) {
    const uint32_t g = first + k * stride;
    if (g < total) fetch(k, g);
    cp_async_commit();
  }
  cp_async_wait<kAddSlots - 1>();  // the table group has landed (for this thread's part)
  __syncthreads();                 // ... and for every thread's part
  int slot = 0;
  for (uint32_t g = first; g < total; g += stride) {
    const uint32_t ahead = g + (kAddSlots - 1) * stride;
    const int refill = slot == 0 ? kAddSlots - 1 : slot - 1;  // the slot used last iteration
    if (ahead < total) fetch(refill, ahead);
    cp_async_commit();
    cp_async_wait<kAddSlots - 1>();  // the group that filled `slot`
    const uint4 v = lut_vec(lut, ring_r[slot * kLutThreads]);
    const uint4 u = ring_a[slot * kLutThreads];
    const uint32_t row = rows.vpr.div(g), col = g - row * rows.vpr.d;
    *reinterpret_cast<uint4*>(y + (int64_t)row * rows.ys + (int64_t)col * 8) =
        make_uint4(add_word(u.x, v.x), add_word(u.y, v.y), add_word(u.z, v.z), add_word(u.w, v.w));
    slot = slot == kAddSlots - 1 ? 0 : slot + 1;
  }
  cp_async_wait<0>();
}

template <int K>
ttn_status rows2(const uint16_t* x, int64_t xs1, int64_t xs2, uint16_t* y, int64_t ys1, int64_t ys2,
                 int64_t n1, int64_t n2, int64_t ncols, cudaStream_t s) {
  const int64_t vpr = ncols / 8, total = n1 * n2 * vpr;
  if (total >= kLutMinVecs && total < ((int64_t)1 << 31)) {
    LutRows rows{xs1, xs2, ys1, ys2, FastDiv((uint32_t)vpr), FastDiv((uint32_t)n2)};
    return launch_lut<true>(K, x, y, rows, total, nullptr, nullptr, 0, s, "unary_rows2_f16");
  }
  // arithmetic rows kernel; its queue holds 32-bit element offsets from y, so
  // each launch covers a slice of i1 whose y extent stays below 2^32
  const int64_t extent = (n2 - 1) * ys2 + ncols;
  if (extent >= ((int64_t)1 << 32)) return fail(TTN_UNSUPPORTED, "unary_rows2_f16: row family too wide");
  int64_t per = ys1 > 0 ? (((int64_t)1 << 32) - extent) / ys1 + 1 : n1;
  if (per < 1) per = 1;
  for (int64_t i0 = 0; i0 < n1; i0 += per) {
    const int64_t m1 = n1 - i0 < per ? n1 - i0 : per;
    Index6 ix;
    ix.ndim = 2;
    ix.size[0] = n2;
    ix.size[1] = m1;
    ix.stride[0][0] = xs2;
    ix.stride[0][1] = xs1;
    ix.stride[1][0] = ys2;
    ix.stride[1][1] = ys1;
    ix.stride[2][0] = ix.stride[2][1] = 0;
    const int64_t rows = m1 * n2;
    int64_t cap = (int64_t)sm_count() * resident_blocks((const void*)unary_f16_vec<K>, kThreads, 0);
    int64_t gy = rows < 65535 ? rows : 65535;
    int64_t gx = (vpr + kThreads * kVec - 1) / (kThreads * kVec);
    int64_t fit = (cap + gy - 1) / gy;
    if (gx > fit) gx = fit;
    if (gx < 1) gx = 1;
    unary_f16_vec<K><<<dim3((unsigned)gx, (unsigned)gy), kThreads, 0, s>>>(x + i0 * xs1, y + i0 * ys1, ix,
                                                                          vpr, rows);
    TTN_TRY(launch_check("unary_rows2_f16"));
  }
  return TTN_OK;
}

// Any layout (also unaligned dense), one element per thread.
template <int K, typename T>
__global__ void __launch_bounds__(kThreads) unary_strided(const T* x, T* y, Index6 ix, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t ox, oy, unused;
    offsets3(ix, i, ox, oy, unused);
    if constexpr (sizeof(T) == 2) {
      reinterpret_cast<uint16_t*>(y)[oy] = unary_h<K>(reinterpret_cast<const uint16_t*>(x)[ox]);
    } else {
      y[oy] = unary_f<K>(x[ox]);
    }
  }
}

// Rows of dense fp16 (e.g. channel-block chunks of NC1HWC0 batches): the
// innermost coalesced dim is unit-stride with a multiple of 8 elements and
// every outer stride is a multiple of 8, so 16-byte vectors still apply.
// ---------------------------------------------------------------- binary

// CPU eager semantics per op (FP32 opmath, x86 IEEE): add/sub use one rounding
// of x +- y when alpha == 1, and fma(y, +-alpha, x) otherwise (the vectorised
// fmadd of the ATen CPU kernel); mul and div are single IEEE operations.
struct BinaryParams {
  int op;
  float alpha;
};

__device__ __forceinline__ float binary_f(const BinaryParams& p, float a, float b) {
  switch (p.op) {
    case TTN_ADD: return p.alpha == 1.0f ? __fadd_rn(a, b) : __fmaf_rn(b, p.alpha, a);
    case TTN_SUB: return p.alpha == 1.0f ? __fsub_rn(a, b) : __fmaf_rn(b, -p.alpha, a);
    case TTN_MUL: return __fmul_rn(a, b);
    default: return __fdiv_rn(a, b);
  }
}

__device__ __forceinline__ uint32_t binary_h2(const BinaryParams& p, uint32_t a, uint32_t b) {
  __half2 ha = *reinterpret_cast<__half2*>(&a);
  __half2 hb = *reinterpret_cast<__half2*>(&b);
  float2 fa = __half22float2(ha), fb = __half22float2(hb);
  __half2 r = __floats2half2_rn(binary_f(p, fa.x, fb.x), binary_f(p, fa.y, fb.y));
  return *reinterpret_cast<uint32_t*>(&r);
}

__global__ void __launch_bounds__(kThreads) binary_f16_dense(BinaryParams p, const uint4* x,
                                                             const uint4* y, uint4* z,
                                                             int64_t nvec, const uint16_t* xt,
                                                             const uint16_t* yt, uint16_t* zt,
                                                             int tail) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    uint4 a = x[i], b = y[i];
    uint4 r;
    r.x = binary_h2(p, a.x, b.x);
    r.y = binary_h2(p, a.y, b.y);
    r.z = binary_h2(p, a.z, b.z);
    r.w = binary_h2(p, a.w, b.w);
    z[i] = r;
  }
  if (blockIdx.x == 0 && (int)threadIdx.x < tail) {
    float a = __half2float(hfrom(xt[threadIdx.x])), b = __half2float(hfrom(yt[threadIdx.x]));
    zt[threadIdx.x] = hbits(__float2half_rn(binary_f(p, a, b)));
  }
}

__global__ void __launch_bounds__(kThreads) binary_f16_rows(BinaryParams p, const uint16_t* x,
                                                            const uint16_t* y, uint16_t* z,
                                                            Index6 outer, int64_t vec_per_row,
                                                            int64_t rows) {
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    int64_t ox, oy, oz;
    offsets3(outer, row, ox, oy, oz);  // once per block row
    const uint4* xs = reinterpret_cast<const uint4*>(x + ox);
    const uint4* ys = reinterpret_cast<const uint4*>(y + oy);
    uint4* zs = reinterpret_cast<uint4*>(z + oz);
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < vec_per_row;
         v += (int64_t)gridDim.x * blockDim.x) {
      uint4 a = xs[v], b = ys[v];
      uint4 r;
      r.x = binary_h2(p, a.x, b.x);
      r.y = binary_h2(p, a.y, b.y);
      r.z = binary_h2(p, a.z, b.z);
      r.w = binary_h2(p, a.w, b.w);
      zs[v] = r;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) binary_strided(BinaryParams p, const T* x, const T* y,
                                                           T* z, Index6 ix, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t ox, oy, oz;
    offsets3(ix, i, ox, oy, oz);
    if constexpr (sizeof(T) == 2) {
      float a = __half2float(x[ox]), b = __half2float(y[oy]);
      z[oz] = __float2half_rn(binary_f(p, a, b));
    } else {
      z[oz] = binary_f(p, x[ox], y[oy]);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) scalar_strided(BinaryParams p, const T* x, float s,
                                                           T* z, Index6 ix, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t ox, oz, unused;
    offsets3(ix, i, ox, oz, unused);
    if constexpr (sizeof(T) == 2) {
      z[oz] = __float2half_rn(binary_f(p, __half2float(x[ox]), s));
    } else {
      z[oz] = binary_f(p, x[ox], s);
    }
  }
}

__global__ void __launch_bounds__(kThreads) scalar_f16_dense(BinaryParams p, const uint4* x,
                                                             float s, uint4* z, int64_t nvec,
                                                             const uint16_t* xt, uint16_t* zt,
                                                             int tail) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    uint4 a = x[i];
    uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __half2 h = *reinterpret_cast<__half2*>(&w[k]);
      float2 f = __half22float2(h);
      __half2 r = __floats2half2_rn(binary_f(p, f.x, s), binary_f(p, f.y, s));
      w[k] = *reinterpret_cast<uint32_t*>(&r);
    }
    z[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (blockIdx.x == 0 && (int)threadIdx.x < tail)
    zt[threadIdx.x] =
        hbits(__float2half_rn(binary_f(p, __half2float(hfrom(xt[threadIdx.x])), s)));
}

// ------------------------------------------- fused SiLU(x + b) + r, NC1HWC0

// x, r, y: [n, c1, hw, 16] fp16; b: [c1*16].  Each uint4 covers half of one
// pixel's 16 channel lanes, so its 8 bias values are contiguous in b.
__device__ __forceinline__ uint4 bias_silu_residual_vec(uint4 xv, uint4 rv, uint4 bv) {
  uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
  uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
  uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
  uint32_t out[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float2 fx = __half22float2(*reinterpret_cast<__half2*>(&xw[k]));
    float2 fr = __half22float2(*reinterpret_cast<__half2*>(&rw[k]));
    float2 fb = __half22float2(*reinterpret_cast<__half2*>(&bw[k]));
    float lo = silu_fast_f32(fx.x + fb.x) + fr.x;
    float hi = silu_fast_f32(fx.y + fb.y) + fr.y;
    __half2 h = __floats2half2_rn(lo, hi);
    out[k] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// nvec 16-byte vectors (< 2^31) starting at plane p0; a plane is one (image,
// channel block) of hw pixels = 2*hw vectors, and its bias block is
// (p0 + plane) mod c1.  Two vectors per thread per step.
__global__ void __launch_bounds__(kThreads) bias_silu_residual(const uint4* x, const uint16_t* b,
                                                               const uint4* r, uint4* y, uint32_t nvec,
                                                               FastDiv vec_per_plane, FastDiv c1,
                                                               uint32_t p0) {
  const uint32_t stride = gridDim.x * blockDim.x;
  auto bias_of = [&](uint32_t i) {
    const uint32_t plane = vec_per_plane.div(i) + p0;
    const uint32_t block = plane - c1.div(plane) * c1.d;
    return *reinterpret_cast<const uint4*>(b + block * 16 + (i & 1) * 8);
  };
  uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + stride < nvec; i += 2 * stride) {
    const uint4 x0 = x[i], r0 = r[i], x1 = x[i + stride], r1 = r[i + stride];
    y[i] = bias_silu_residual_vec(x0, r0, bias_of(i));
    y[i + stride] = bias_silu_residual_vec(x1, r1, bias_of(i + stride));
  }
  if (i < nvec) y[i] = bias_silu_residual_vec(x[i], r[i], bias_of(i));
}

// ----------------------------------------------------------- host helpers

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// Dense when every view is contiguous with identical element order.
bool dense(const Coalesced& c, int count) {
  if (c.ndim > 1) return false;
  if (c.ndim == 0) return true;
  for (int v = 0; v < count; ++v)
    if (c.stride[v][0] != 1) return false;
  return true;
}

// Vectorisable rows: unit inner stride, inner length and outer strides in
// multiples of 8 elements, 16-byte aligned bases, at most 6 outer dims.
bool vec_rows(const Coalesced& c, int count, const void* const* ptrs, Index6& outer,
              int64_t& vec_per_row) {
  if (c.ndim < 2 || c.ndim > 7 || c.size[0] % 8) return false;
  for (int v = 0; v < count; ++v) {
    if (c.stride[v][0] != 1 || ((uintptr_t)ptrs[v] & 15u)) return false;
    for (int d = 1; d < c.ndim; ++d)
      if (c.stride[v][d] % 8) return false;
  }
  outer.ndim = c.ndim - 1;
  for (int d = 0; d < 6; ++d) {
    outer.size[d] = d + 1 < c.ndim ? c.size[d + 1] : 1;
    for (int v = 0; v < 3; ++v)
      outer.stride[v][d] = (d + 1 < c.ndim && v < count) ? c.stride[v][d + 1] : 0;
  }
  vec_per_row = c.size[0] / 8;
  return true;
}

// True when the largest element offset of operand v is below 2^32.
bool extent_below_2_32(const Coalesced& c, int v) {
  int64_t extent = 0;
  for (int d = 0; d < c.ndim; ++d) extent += (c.size[d] - 1) * (c.stride[v][d] < 0 ? -c.stride[v][d] : c.stride[v][d]);
  return extent < ((int64_t)1 << 32) - 8;
}

// 2-D grid for row kernels: y over rows (<= 65535 per pass), x over the
// vectors of a row, about 8 resident blocks per SM in total.
dim3 rows_grid(int64_t vec_per_row, int64_t rows) {
  int64_t gy = rows < 65535 ? rows : 65535;
  int64_t want = (int64_t)sm_count() * 8;
  int64_t gx = (vec_per_row + kThreads - 1) / kThreads;
  int64_t cap = (want + gy - 1) / gy;
  if (gx > cap) gx = cap;
  if (gx < 1) gx = 1;
  return dim3((unsigned)gx, (unsigned)gy);
}

ttn_status to_index6(const Coalesced& c, int count, Index6& ix, const char* what) {
  if (c.ndim > 6)
    return fail(TTN_UNSUPPORTED, "%s: view needs %d dims after coalescing (max 6)", what, c.ndim);
  ix.ndim = c.ndim;
  for (int d = 0; d < 6; ++d) {
    ix.size[d] = d < c.ndim ? c.size[d] : 1;
    for (int v = 0; v < 3; ++v) ix.stride[v][d] = (d < c.ndim && v < count) ? c.stride[v][d] : 0;
  }
  return TTN_OK;
}

template <int K>
ttn_status unary(const ttn_tensor* x, const ttn_tensor* y, ttn_stream stream, const char* name) {
  TTN_TRY(validate(x, name));
  TTN_TRY(validate(y, name));
  if (!same_sizes(x, y)) return fail(TTN_INVALID_ARG, "%s: x and y sizes differ", name);
  if (x->dtype != y->dtype) return fail(TTN_INVALID_ARG, "%s: x and y dtypes differ", name);
  const ttn_tensor* views[2] = {x, y};
  Coalesced c = coalesce(views, 2);
  if (!c.numel) return TTN_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (x->dtype == TTN_F16 && dense(c, 2) && aligned16(x->data) && aligned16(y->data)) {
    const int64_t total_vec = c.numel / 8;
    const int tail = (int)(c.numel - total_vec * 8);
    const int64_t chunk = (int64_t)1 << 28;  // vectors per launch: 2^31 elements
    for (int64_t v0 = 0; v0 < total_vec || (v0 == 0 && tail); v0 += chunk) {
      int64_t nvec = total_vec - v0 < chunk ? total_vec - v0 : chunk;
      bool last = v0 + chunk >= total_vec;
      if (nvec >= kLutMinVecs) {
        const LutRows dense_rows{0, 0, 0, 0, FastDiv(1), FastDiv(1)};
        TTN_TRY(launch_lut<false>(K, (const uint16_t*)x->data + v0 * 8, (uint16_t*)y->data + v0 * 8,
                                  dense_rows, nvec, (const uint16_t*)x->data + total_vec * 8,
                                  (uint16_t*)y->data + total_vec * 8, last ? tail : 0, s, name));
      } else {
        unsigned grid = resident_grid(unary_f16_dense<K>, kThreads, 0, nvec ? nvec : 1,
                                      (int64_t)kThreads * kVec);
        TTN_TRY(cuda_check(launch_pdl(unary_f16_dense<K>, dim3(grid), dim3(kThreads), 0, s,
                                      (const uint16_t*)x->data + v0 * 8, (uint16_t*)y->data + v0 * 8, (int)nvec,
                                      (const uint16_t*)x->data + total_vec * 8,
                                      (uint16_t*)y->data + total_vec * 8, last ? tail : 0),
                           name));
      }
      TTN_TRY(launch_check(name));
      if (last) break;
    }
    return TTN_OK;
  }
  if (x->dtype == TTN_F16 && c.ndim >= 2 && c.ndim <= 3 && c.stride[0][0] == 1 && c.stride[1][0] == 1 &&
      c.size[0] % 8 == 0 && aligned16(x->data) && aligned16(y->data) && c.size[1] < ((int64_t)1 << 32) &&
      c.size[0] / 8 < ((int64_t)1 << 32)) {  // rows with up to two outer dims: table or arithmetic
    bool rows16 = true;
    for (int d = 1; d < c.ndim; ++d) rows16 = rows16 && c.stride[0][d] % 8 == 0 && c.stride[1][d] % 8 == 0;
    if (rows16) {
      const bool two = c.ndim == 3;
      ttn_status st = unary_rows2_f16(K, (const uint16_t*)x->data, two ? c.stride[0][2] : 0, c.stride[0][1],
                                      (uint16_t*)y->data, two ? c.stride[1][2] : 0, c.stride[1][1],
                                      two ? c.size[2] : 1, c.size[1], c.size[0], s);
      if (st != TTN_UNSUPPORTED) return st;  // too wide for 32-bit queue offsets: general paths below
    }
  }
  Index6 ix;
  int64_t vpr;
  const void* ptrs[2] = {x->data, y->data};
  if (x->dtype == TTN_F16 && vec_rows(c, 2, ptrs, ix, vpr) && extent_below_2_32(c, 1)) {
    const int64_t rows = c.numel / 8 / vpr;
    int64_t cap = (int64_t)sm_count() * resident_blocks((const void*)unary_f16_vec<K>, kThreads, 0);
    int64_t gy = rows < 65535 ? rows : 65535;
    int64_t gx = (vpr + kThreads * kVec - 1) / (kThreads * kVec);
    int64_t fit = (cap + gy - 1) / gy;
    if (gx > fit) gx = fit;
    if (gx < 1) gx = 1;
    unary_f16_vec<K><<<dim3((unsigned)gx, (unsigned)gy), kThreads, 0, s>>>(
        (const uint16_t*)x->data, (uint16_t*)y->data, ix, vpr, rows);
    return launch_check(name);
  }
  TTN_TRY(to_index6(c, 2, ix, name));
  unsigned grid = grid_for(c.numel, kThreads);
  if (x->dtype == TTN_F16)
    unary_strided<K, __half><<<grid, kThreads, 0, s>>>((const __half*)x->data, (__half*)y->data, ix,
                                                        c.numel);
  else
    unary_strided<K, float><<<grid, kThreads, 0, s>>>((const float*)x->data, (float*)y->data, ix,
                                                       c.numel);
  return launch_check(name);
}

}  // namespace

ttn_status unary_rows2_f16(int kind, const uint16_t* x, int64_t xs1, int64_t xs2, uint16_t* y,
                           int64_t ys1, int64_t ys2, int64_t n1, int64_t n2, int64_t ncols,
                           cudaStream_t stream) {
  if (n1 <= 0 || n2 <= 0 || ncols <= 0) return TTN_OK;
  if (ncols % 8 || xs1 % 8 || xs2 % 8 || ys1 % 8 || ys2 % 8 || !aligned16(x) || !aligned16(y))
    return fail(TTN_INVALID_ARG, "unary_rows2_f16: rows must be 16-byte aligned");
  if (n2 >= ((int64_t)1 << 32) || ncols / 8 >= ((int64_t)1 << 32))
    return fail(TTN_UNSUPPORTED, "unary_rows2_f16: dimension beyond 2^32");
  return kind == kSilu ? rows2<kSilu>(x, xs1, xs2, y, ys1, ys2, n1, n2, ncols, stream)
                       : rows2<kSigmoid>(x, xs1, xs2, y, ys1, ys2, n1, n2, ncols, stream);
}

}  // namespace ttn

using namespace ttn;

extern "C" {

ttn_status ttn_silu(const ttn_tensor* x, const ttn_tensor* y, ttn_stream stream) {
  return unary<kSilu>(x, y, stream, "ttn_silu");
}

ttn_status ttn_sigmoid(const ttn_tensor* x, const ttn_tensor* y, ttn_stream stream) {
  return unary<kSigmoid>(x, y, stream, "ttn_sigmoid");
}

ttn_status ttn_add_silu_f16(const ttn_tensor* a, const ttn_tensor* raw, const ttn_tensor* out,
                            ttn_stream stream) {
  const char* name = "ttn_add_silu_f16";
  TTN_TRY(validate(a, name));
  TTN_TRY(validate(raw, name));
  TTN_TRY(validate(out, name));
  if (!same_sizes(a, raw) || !same_sizes(a, out)) return fail(TTN_INVALID_ARG, "%s: operand sizes differ", name);
  if (a->dtype != TTN_F16 || raw->dtype != TTN_F16 || out->dtype != TTN_F16)
    return fail(TTN_INVALID_ARG, "%s: fp16 operands only", name);
  const ttn_tensor* views[3] = {raw, a, out};
  Coalesced c = coalesce(views, 3);
  if (!c.numel) return TTN_OK;
  // rows of contiguous 16-byte vectors: at most two coalesced dims, unit inner stride
  const bool rows_ok = c.ndim <= 2 && c.stride[0][0] == 1 && c.stride[1][0] == 1 && c.stride[2][0] == 1 &&
                       c.size[0] % 8 == 0 && aligned16(raw->data) && aligned16(a->data) && aligned16(out->data) &&
                       (c.ndim == 1 || (c.stride[0][1] % 8 == 0 && c.stride[1][1] % 8 == 0 && c.stride[2][1] % 8 == 0));
  if (!rows_ok)
    return fail(TTN_UNSUPPORTED, "%s: operands must be rows of 16-byte aligned contiguous vectors", name);
  const int64_t vpr = c.size[0] / 8, n1 = c.ndim == 2 ? c.size[1] : 1, total = n1 * vpr;
  if (total >= ((int64_t)1 << 31) || vpr >= ((int64_t)1 << 32))
    return fail(TTN_UNSUPPORTED, "%s: more than 2^31 vectors", name);
  AddRows rows{c.ndim == 2 ? c.stride[0][1] : 0, c.ndim == 2 ? c.stride[1][1] : 0,
               c.ndim == 2 ? c.stride[2][1] : 0, FastDiv((uint32_t)vpr)};
  cudaStream_t s = (cudaStream_t)stream;
  const uint16_t* table = nullptr;
  TTN_TRY(unary_table(kSilu, s, &table));
  TTN_TRY(ensure_dynamic_smem((const void*)add_silu_lut, kAddSmem));
  const int64_t want = (total + 4 * kLutThreads - 1) / (4 * kLutThreads);
  const unsigned grid = (unsigned)(want < sm_count() ? (want < 1 ? 1 : want) : sm_count());
  TTN_TRY(cuda_check(launch_pdl(add_silu_lut, grid, kLutThreads, kAddSmem, s, table, (const uint16_t*)raw->data,
                                (const uint16_t*)a->data, (uint16_t*)out->data, rows, (uint32_t)total),
                     name));
  return launch_check(name);
}

ttn_status ttn_binary(int op, float alpha, const ttn_tensor* x, const ttn_tensor* y,
                      const ttn_tensor* out, ttn_stream stream) {
  const char* name = "ttn_binary";
  if (op < TTN_SUB || op > TTN_ADD) return fail(TTN_INVALID_ARG, "%s: unknown op %d", name, op);
  TTN_TRY(validate(x, name));
  TTN_TRY(validate(y, name));
  TTN_TRY(validate(out, name));
  if (!same_sizes(x, y) || !same_sizes(x, out))
    return fail(TTN_INVALID_ARG, "%s: operand sizes differ (expand broadcasts first)", name);
  if (x->dtype != y->dtype || x->dtype != out->dtype)
    return fail(TTN_INVALID_ARG, "%s: operand dtypes differ", name);
  const ttn_tensor* views[3] = {x, y, out};
  Coalesced c = coalesce(views, 3);
  if (!c.numel) return TTN_OK;
  BinaryParams p{op, alpha};
  cudaStream_t s = (cudaStream_t)stream;
  if (x->dtype == TTN_F16 && dense(c, 3) && aligned16(x->data) && aligned16(y->data) &&
      aligned16(out->data)) {
    int64_t nvec = c.numel / 8;
    int tail = (int)(c.numel - nvec * 8);
    unsigned grid = grid_for(nvec ? nvec : 1, kThreads);
    binary_f16_dense<<<grid, kThreads, 0, s>>>(
        p, (const uint4*)x->data, (const uint4*)y->data, (uint4*)out->data, nvec,
        (const uint16_t*)x->data + nvec * 8, (const uint16_t*)y->data + nvec * 8,
        (uint16_t*)out->data + nvec * 8, tail);
    return launch_check(name);
  }
  Index6 ix;
  int64_t vpr;
  const void* ptrs[3] = {x->data, y->data, out->data};
  if (x->dtype == TTN_F16 && vec_rows(c, 3, ptrs, ix, vpr)) {
    dim3 grid = rows_grid(vpr, c.numel / 8 / vpr);
    binary_f16_rows<<<grid, kThreads, 0, s>>>(p, (const uint16_t*)x->data, (const uint16_t*)y->data,
                                              (uint16_t*)out->data, ix, vpr, c.numel / 8 / vpr);
    return launch_check(name);
  }
  TTN_TRY(to_index6(c, 3, ix, name));
  unsigned grid = grid_for(c.numel, kThreads);
  if (x->dtype == TTN_F16)
    binary_strided<__half><<<grid, kThreads, 0, s>>>(p, (const __half*)x->data,
                                                      (const __half*)y->data, (__half*)out->data,
                                                      ix, c.numel);
  else
    binary_strided<float><<<grid, kThreads, 0, s>>>(p, (const float*)x->data, (const float*)y->data,
                                                     (float*)out->data, ix, c.numel);
  return launch_check(name);
}

ttn_status ttn_binary_scalar(int op, double scalar, const ttn_tensor* x, const ttn_tensor* out,
                             ttn_stream stream) {
  const char* name = "ttn_binary_scalar";
  if (op < TTN_SUB || op > TTN_ADD) return fail(TTN_INVALID_ARG, "%s: unknown op %d", name, op);
  TTN_TRY(validate(x, name));
  TTN_TRY(validate(out, name));
  if (!same_sizes(x, out)) return fail(TTN_INVALID_ARG, "%s: sizes differ", name);
  if (x->dtype != out->dtype) return fail(TTN_INVALID_ARG, "%s: dtypes differ", name);
  const ttn_tensor* views[2] = {x, out};
  Coalesced c = coalesce(views, 2);
  if (!c.numel) return TTN_OK;
  BinaryParams p{op, 1.0f};
  float s32 = (float)scalar;
  cudaStream_t s = (cudaStream_t)stream;
  if (x->dtype == TTN_F16 && dense(c, 2) && aligned16(x->data) && aligned16(out->data)) {
    int64_t nvec = c.numel / 8;
    int tail = (int)(c.numel - nvec * 8);
    unsigned grid = grid_for(nvec ? nvec : 1, kThreads);
    scalar_f16_dense<<<grid, kThreads, 0, s>>>(p, (const uint4*)x->data, s32, (uint4*)out->data,
                                               nvec, (const uint16_t*)x->data + nvec * 8,
                                               (uint16_t*)out->data + nvec * 8, tail);
    return launch_check(name);
  }
  Index6 ix;
  TTN_TRY(to_index6(c, 2, ix, name));
  unsigned grid = grid_for(c.numel, kThreads);
  if (x->dtype == TTN_F16)
    scalar_strided<__half><<<grid, kThreads, 0, s>>>(p, (const __half*)x->data, s32,
                                                      (__half*)out->data, ix, c.numel);
  else
    scalar_strided<float><<<grid, kThreads, 0, s>>>(p, (const float*)x->data, s32,
                                                     (float*)out->data, ix, c.numel);
  return launch_check(name);
}

ttn_status ttn_bias_silu_residual_nc1hwc0_f16(const void* x, const void* bias,
                                              const void* residual, void* y, int64_t n,
                                              int64_t c1, int64_t hw, ttn_stream stream) {
  const char* name = "ttn_bias_silu_residual_nc1hwc0_f16";
  if (n < 0 || c1 < 0 || hw < 0) return fail(TTN_INVALID_ARG, "%s: negative size", name);
  int64_t count = n * c1 * hw * 16;
  if (!count) return TTN_OK;
  if (!x || !bias || !residual || !y) return fail(TTN_INVALID_ARG, "%s: null pointer", name);
  if (!aligned16(x) || !aligned16(bias) || !aligned16(residual) || !aligned16(y))
    return fail(TTN_INVALID_ARG, "%s: pointers must be 16-byte aligned", name);
  // launches of whole planes, each below 2^31 vectors (32-bit index math)
  const int64_t vpp = 2 * hw, planes = n * c1;
  if (vpp >= ((int64_t)1 << 31) || c1 >= ((int64_t)1 << 31))
    return fail(TTN_UNSUPPORTED, "%s: plane beyond 2^31 vectors", name);
  const int64_t per = (((int64_t)1 << 31) - 1) / vpp;
  for (int64_t p = 0; p < planes; p += per) {
    const int64_t m = planes - p < per ? planes - p : per;
    const int64_t nvec = m * vpp;
    unsigned grid = grid_for(nvec, 2 * kThreads);
    bias_silu_residual<<<grid, kThreads, 0, (cudaStream_t)stream>>>(
        (const uint4*)x + p * vpp, (const uint16_t*)bias, (const uint4*)residual + p * vpp,
        (uint4*)y + p * vpp, (uint32_t)nvec, FastDiv((uint32_t)vpp), FastDiv((uint32_t)c1),
        (uint32_t)(p % c1));
    TTN_TRY(launch_check(name));
  }
  return TTN_OK;
}

}  // extern "C"
