// YOLO26 NMS-free detection selection (reference: selection_flow.cpp:429-491).
//
// Total order (selection_flow.cpp:30-35, 54-57; selection_sort.h:85-89): a
// score's key is 0 for NaN (or 0xffff with TTN_SELECT_NAN_LAST), 0x7fff for
// +-0, the raw bits for negatives and 0x7fff - bits for positives; smaller
// keys rank first and equal keys keep the lower source index.  That order is
// torch.argsort(descending=True, stable=True) over fp16 scores.
//
// Pipeline per call (b images, a anchors, nc classes, k = min(max_det, a)):
//   1. class_max_*   one pass over the scores: per anchor the first class with
//                    the smallest key -> 32-bit record (score bits | class<<16).
//   2. topk_block    one CTA per image: 16-bit radix select of the k-th key,
//                    index-ordered collection of the k winners (keys below the
//                    threshold plus the lowest-index ties), bitonic sort of the
//                    (key<<32 | index) composites in shared memory.  k > 4096
//                    takes a stable counting sort of every key instead.
//   3. gather_pairs  (class-aware) the k x nc scores of the stage-1 anchors,
//                    then topk_block again over the k*nc flat (rank*nc + class).
//   4. pack          FP32 rows (box bits widened exactly, score, class) and the
//                    optional trace outputs.
// Scratch lives in the caller's workspace (ttn_select_workspace_size).
#include <type_traits>

#include "common.cuh"

namespace ttn {
namespace {

constexpr int kTopkThreads = 1024;
constexpr int kSmemSort = 4096;  // largest k sorted in shared memory
constexpr uint32_t kInvalidKey = 0x10000u;

struct SelectView {
  const uint16_t* base;  // element [0,0,0]
  int64_t sb, sa, sc;    // strides in elements
  int64_t batch, anchors, classes;
};

__device__ __forceinline__ uint32_t score_key(uint16_t bits, bool nan_last) {
  uint32_t magnitude = bits & 0x7fffu;
  if (magnitude > 0x7c00u) return nan_last ? 0xffffu : 0u;
  if (magnitude == 0) return 0x7fffu;
  return (bits & 0x8000u) ? bits : (uint32_t)((~(bits ^ 0x8000u)) & 0xffffu);
}

__device__ __forceinline__ uint16_t score_bits(const SelectView& v, int64_t b, int64_t a, int64_t c,
                                               bool sigmoid) {
  uint16_t raw = v.base[b * v.sb + a * v.sa + (c + 4) * v.sc];
  return sigmoid ? sigmoid_h_fast(raw) : raw;
}

// Per-image histograms of key high bytes kept in global memory: lanes adding to
// the same slot are combined first (one atomic per distinct slot per warp step);
// `live` lanes take part, all lanes of the warp call.
__device__ __forceinline__ void hist_add_global(uint32_t* hist, uint32_t slot, bool live) {
  const uint32_t mask = __ballot_sync(0xffffffffu, live);
  if (!live) return;
  const uint32_t peers = __match_any_sync(mask, slot);
  if ((threadIdx.x & 31) == (uint32_t)(__ffs(peers) - 1)) atomicAdd(&hist[slot], (uint32_t)__popc(peers));
}

// ------------------------------------------------------------ 1. class max

// Thread per anchor (coalesced when anchors are the unit-stride dim).
__global__ void __launch_bounds__(256) class_max_thread(SelectView v, bool nan_last, bool sigmoid,
                                                        uint32_t* records, int64_t rec_pitch,
                                                        uint16_t* trace_max) {
  const int64_t total = v.batch * v.anchors;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    int64_t b = t / v.anchors, a = t % v.anchors;
    uint32_t best = kInvalidKey, best_bits = 0, best_cls = 0;
    const uint16_t* p = v.base + b * v.sb + a * v.sa + 4 * v.sc;
    for (int64_t c = 0; c < v.classes; ++c) {
      uint16_t bits = p[c * v.sc];
      if (sigmoid) bits = sigmoid_h_fast(bits);
      uint32_t key = score_key(bits, nan_last);
      if (key < best) {
        best = key;
        best_bits = bits;
        best_cls = (uint32_t)c;
      }
    }
    records[b * rec_pitch + a] = best_bits | (best_cls << 16);
    if (trace_max) trace_max[t] = (uint16_t)best_bits;
  }
}

// Channel-planar scores (anchor stride 1, 16-byte aligned rows): 8 anchors per
// thread with 128-bit loads, one class row at a time.
__global__ void __launch_bounds__(256) class_max_planar8(SelectView v, bool nan_last, bool sigmoid,
                                                         uint32_t* records, int64_t rec_pitch,
                                                         uint16_t* trace_max) {
  const int64_t groups = v.anchors / 8;
  const int64_t total = v.batch * groups;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    int64_t b = t / groups, a0 = (t % groups) * 8;
    uint32_t best[8], bits8[8], cls8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      best[j] = kInvalidKey;
      bits8[j] = 0;
      cls8[j] = 0;
    }
    const uint16_t* p = v.base + b * v.sb + a0 + 4 * v.sc;
    int64_t c = 0;
    for (; c + 1 < v.classes; c += 2) {  // two rows in flight
      uint4 q0 = *reinterpret_cast<const uint4*>(p + c * v.sc);
      uint4 q1 = *reinterpret_cast<const uint4*>(p + (c + 1) * v.sc);
      uint32_t w[2][4] = {{q0.x, q0.y, q0.z, q0.w}, {q1.x, q1.y, q1.z, q1.w}};
#pragma unroll
      for (int r = 0; r < 2; ++r) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint16_t bits = (uint16_t)((w[r][j >> 1] >> ((j & 1) * 16)) & 0xffffu);
          if (sigmoid) bits = sigmoid_h_fast(bits);
          uint32_t key = score_key(bits, nan_last);
          if (key < best[j]) {
            best[j] = key;
            bits8[j] = bits;
            cls8[j] = (uint32_t)(c + r);
          }
        }
      }
    }
    if (c < v.classes) {
      uint4 q0 = *reinterpret_cast<const uint4*>(p + c * v.sc);
      uint32_t w[4] = {q0.x, q0.y, q0.z, q0.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint16_t bits = (uint16_t)((w[j >> 1] >> ((j & 1) * 16)) & 0xffffu);
        if (sigmoid) bits = sigmoid_h_fast(bits);
        uint32_t key = score_key(bits, nan_last);
        if (key < best[j]) {
          best[j] = key;
          bits8[j] = bits;
          cls8[j] = (uint32_t)c;
        }
      }
    }
    uint32_t out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = bits8[j] | (cls8[j] << 16);
    uint4* dst = reinterpret_cast<uint4*>(records + b * rec_pitch + a0);
    dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
    dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
    if (trace_max) {
#pragma unroll
      for (int j = 0; j < 8; ++j) trace_max[b * v.anchors + a0 + j] = (uint16_t)bits8[j];
    }
  }
}

// Fused-sigmoid class max (TTN_SELECT_SIGMOID), planar scores.  fp16 sigmoid
// is monotone non-decreasing, so the best sigmoid belongs to the best logit; only
// ties in the *sigmoid* value can move the winner to a lower class index
// (distinct logits that round to one fp16 sigmoid).  Pass 1 keeps the best and
// second-best logit per anchor (no sigmoid at all); the winner is final unless
// sigmoid(second) equals sigmoid(best), in which case the warp rescans that
// anchor's classes with the exact sigmoid, lanes over classes.
__device__ __forceinline__ void rescan_anchor(const SelectView& v, int64_t b, int64_t a, bool nan_last,
                                              uint32_t& out_bits, uint32_t& out_cls, uint32_t& out_second) {
  const int lane = threadIdx.x & 31;
  const uint16_t* p = v.base + b * v.sb + a * v.sa + 4 * v.sc;
  // best (key, class, bits) and the smallest key among the other classes
  uint32_t best = kInvalidKey, best_cls = 0xffffffffu, best_bits = 0, second = kInvalidKey;
  for (int64_t c = lane; c < v.classes; c += 32) {
    uint16_t bits = sigmoid_h_fast(p[c * v.sc]);
    uint32_t key = score_key(bits, nan_last);
    if (key < best) {
      second = best;
      best = key;
      best_cls = (uint32_t)c;
      best_bits = bits;
    } else {
      second = min(second, key);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    uint32_t ok = __shfl_xor_sync(0xffffffffu, best, o);
    uint32_t oc = __shfl_xor_sync(0xffffffffu, best_cls, o);
    uint32_t ob = __shfl_xor_sync(0xffffffffu, best_bits, o);
    uint32_t os = __shfl_xor_sync(0xffffffffu, second, o);
    if (ok < best || (ok == best && oc < best_cls)) {
      second = min(os, best);
      best = ok;
      best_cls = oc;
      best_bits = ob;
    } else {
      second = min(second, ok);
    }
  }
  out_bits = best_bits;
  out_cls = best_cls;
  out_second = min(second, 0xffffu);
}

// Pass 1 works on the fp16 logits two anchors at a time (half2 lanes), since
// fp16 sigmoid is monotonic: per class row, best = max(best, x) and second =
// max(second, min(best, x)) (packed fp16 max/min), and the class moves only on
// a strictly greater logit (a packed compare mask and one 3-input logic op), so
// the first class of the largest logit is kept.  An inf or NaN logit makes
// x * 0 NaN in a per-lane accumulator.  Anchors with such a logit, or whose
// best and second-best logits give the same fp16 sigmoid (this also covers
// +0/-0 and equal logits), are decided by the exact rescan.
// APT anchors per thread (2, 4 or 8: 4-, 8- or 16-byte loads per class row),
// 32/APT class rows in flight per thread.
template <int APT>
__global__ void __launch_bounds__(256) class_max_planar_sigmoid(SelectView v, bool nan_last,
                                                                uint32_t* records, int64_t rec_pitch,
                                                                uint16_t* trace_max, uint16_t* second_keys,
                                                                uint32_t* key_hist) {
  constexpr int W = APT / 2;      // half2 words per class row
  constexpr int ROWS = 64 / APT;  // class rows in flight
  using Vec = typename std::conditional<W == 4, uint4, typename std::conditional<W == 2, uint2, uint32_t>::type>::type;
  const int lane = threadIdx.x & 31;
  const int64_t groups = v.anchors / APT;
  const int64_t total = v.batch * groups;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const __half2 zero = __float2half2_rn(0.0f);
  const __half2 neg_inf = __halves2half2(__ushort_as_half(0xfc00u), __ushort_as_half(0xfc00u));
  // warp-uniform trip count so the rescan can use the whole warp
  for (int64_t t0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31); t0 < total; t0 += stride) {
    const int64_t t = t0 + lane;
    const bool live = t < total;
    const int64_t b = live ? t / groups : 0, a0 = live ? (t % groups) * APT : 0;
    __half2 best[W], second[W], special[W];
    uint32_t cls[W];
#pragma unroll
    for (int k = 0; k < W; ++k) {
      best[k] = second[k] = neg_inf;
      special[k] = zero;
      cls[k] = 0;
    }
    if (live) {
      const uint16_t* p = v.base + b * v.sb + a0 + 4 * v.sc;
      auto fold = [&](const Vec q, uint32_t c) {
        const uint32_t cpair = c * 0x00010001u;
        const uint32_t* w = reinterpret_cast<const uint32_t*>(&q);
#pragma unroll
        for (int k = 0; k < W; ++k) {
          const __half2 x = *reinterpret_cast<const __half2*>(&w[k]);
          const uint32_t m = __hgt2_mask(x, best[k]);
          cls[k] = (cls[k] & ~m) | (cpair & m);
          second[k] = __hmax2(second[k], __hmin2(best[k], x));
          best[k] = __hmax2(best[k], x);
          special[k] = __hfma2(x, zero, special[k]);
        }
      };
      int64_t c = 0;
      for (; c + ROWS - 1 < v.classes; c += ROWS) {  // ROWS class rows in flight
        Vec q[ROWS];
#pragma unroll
        for (int u = 0; u < ROWS; ++u) q[u] = *reinterpret_cast<const Vec*>(p + (c + u) * v.sc);
#pragma unroll
        for (int u = 0; u < ROWS; ++u) fold(q[u], (uint32_t)(c + u));
      }
      for (; c < v.classes; ++c) fold(*reinterpret_cast<const Vec*>(p + c * v.sc), (uint32_t)c);
    }
    uint32_t out_bits[APT], clsj[APT], redo = 0;
    uint32_t skey[APT];  // key of the best score among the other classes (0xffff: none)
#pragma unroll
    for (int j = 0; j < APT; ++j) {
      const int k = j >> 1, sh = (j & 1) * 16;
      const uint16_t logit = (uint16_t)(*reinterpret_cast<const uint32_t*>(&best[k]) >> sh);
      const uint16_t flag = (uint16_t)(*reinterpret_cast<const uint32_t*>(&special[k]) >> sh);
      clsj[j] = (cls[k] >> sh) & 0xffffu;
      const uint16_t s1 = sigmoid_h_fast(logit);
      out_bits[j] = s1;
      const bool has_special = (flag & 0x7fffu) > 0x7c00u;  // NaN: some logit was inf or NaN
      bool tie = false;
      skey[j] = 0xffffu;
      if (v.classes > 1) {  // sigmoid is monotonic: the second logit gives the second score
        const uint16_t s2 = sigmoid_h_fast((uint16_t)(*reinterpret_cast<const uint32_t*>(&second[k]) >> sh));
        skey[j] = score_key(s2, nan_last);
        tie = skey[j] == score_key(s1, nan_last);
      }
      // A tie can only move the winner to a lower class index, so an anchor whose
      // first largest logit is class 0 keeps it (e.g. a row of equal logits).
      if (live && (has_special || (tie && clsj[j] != 0))) redo |= 1u << j;
    }
    // exact rescans, one anchor at a time with the whole warp
    uint32_t pending = __ballot_sync(0xffffffffu, redo != 0);
    while (pending) {
      const int src = __ffs(pending) - 1;
      uint32_t src_redo = __shfl_sync(0xffffffffu, redo, src);
      const int64_t sb = __shfl_sync(0xffffffffu, b, src), sa0 = __shfl_sync(0xffffffffu, a0, src);
      while (src_redo) {
        const int j = __ffs(src_redo) - 1;
        src_redo &= src_redo - 1;
        uint32_t rb, rc, rs;
        rescan_anchor(v, sb, sa0 + j, nan_last, rb, rc, rs);
        if (lane == src) {
#pragma unroll
          for (int k = 0; k < APT; ++k)
            if (k == j) {
              out_bits[k] = rb;
              clsj[k] = rc;
              skey[k] = rs;
            }
        }
      }
      pending &= pending - 1;
    }
    if (key_hist) {  // [b][256] counts of the anchors' best-key high bytes, for the stage-1 top-k
#pragma unroll
      for (int j = 0; j < APT; ++j)
        hist_add_global(key_hist, (uint32_t)b * 256u + (score_key((uint16_t)out_bits[j], nan_last) >> 8), live);
    }
    if (live) {
      uint32_t out[APT];
#pragma unroll
      for (int j = 0; j < APT; ++j) out[j] = out_bits[j] | (clsj[j] << 16);
      if constexpr (APT >= 4) {
        uint4* dst = reinterpret_cast<uint4*>(records + b * rec_pitch + a0);
#pragma unroll
        for (int h = 0; h < APT / 4; ++h)
          dst[h] = make_uint4(out[4 * h], out[4 * h + 1], out[4 * h + 2], out[4 * h + 3]);
      } else {
        *reinterpret_cast<uint2*>(records + b * rec_pitch + a0) = make_uint2(out[0], out[1]);
      }
      if (trace_max) {
#pragma unroll
        for (int j = 0; j < APT; ++j) trace_max[b * v.anchors + a0 + j] = (uint16_t)out_bits[j];
      }
      if (second_keys) {
        uint32_t sw[W];
#pragma unroll
        for (int k = 0; k < W; ++k) sw[k] = skey[2 * k] | (skey[2 * k + 1] << 16);
        *reinterpret_cast<Vec*>(second_keys + b * v.anchors + a0) = *reinterpret_cast<const Vec*>(sw);
      }
    }
  }
}

// Class-contiguous rows (class stride 1): one warp per anchor, lanes over
// classes, (key, class) lexicographic warp reduction.
__global__ void __launch_bounds__(256) class_max_warp(SelectView v, bool nan_last, bool sigmoid,
                                                      uint32_t* records, int64_t rec_pitch,
                                                      uint16_t* trace_max) {
  const int lane = threadIdx.x & 31;
  const int64_t total = v.batch * v.anchors;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < total; t += warps) {
    int64_t b = t / v.anchors, a = t % v.anchors;
    const uint16_t* p = v.base + b * v.sb + a * v.sa + 4 * v.sc;
    uint32_t best = kInvalidKey, best_cls = 0xffffffffu, best_bits = 0;
    for (int64_t c = lane; c < v.classes; c += 32) {
      uint16_t bits = p[c * v.sc];
      if (sigmoid) bits = sigmoid_h_fast(bits);
      uint32_t key = score_key(bits, nan_last);
      if (key < best) {  // lanes walk classes in increasing order
        best = key;
        best_cls = (uint32_t)c;
        best_bits = bits;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      uint32_t ok = __shfl_xor_sync(0xffffffffu, best, o);
      uint32_t oc = __shfl_xor_sync(0xffffffffu, best_cls, o);
      uint32_t ob = __shfl_xor_sync(0xffffffffu, best_bits, o);
      if (ok < best || (ok == best && oc < best_cls)) {
        best = ok;
        best_cls = oc;
        best_bits = ob;
      }
    }
    if (lane == 0) {
      if (best_cls == 0xffffffffu) best_cls = 0;
      records[b * rec_pitch + a] = best_bits | (best_cls << 16);
      if (trace_max) trace_max[t] = (uint16_t)best_bits;
    }
  }
}

// ------------------------------------------------------------- 2. top-k

// Key source for topk_block: stage 1 reads 32-bit records, stage 2 16-bit bits.
struct KeySource {
  const uint32_t* records;  // stage 1 (low 16 bits are the score bits)
  const uint16_t* bits;     // stage 2
  int64_t pitch;            // elements between images
  __device__ __forceinline__ uint16_t get(int64_t b, int64_t i) const {
    return records ? (uint16_t)(records[b * pitch + i] & 0xffffu) : bits[b * pitch + i];
  }
};

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Block-wide exclusive prefix of a per-thread 0/1 flag over threads in order.
// Returns this thread's prefix; *total receives the block total.  Uses
// scratch[32] and synchronises.
__device__ __forceinline__ int block_prefix(bool flag, int* scratch, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t mask = __ballot_sync(0xffffffffu, flag);
  int in_warp = __popc(mask & lanemask_lt());
  if (lane == 0) scratch[warp] = __popc(mask);
  __syncthreads();
  int warps = blockDim.x >> 5;
  if (warp == 0) {
    int v = lane < warps ? scratch[lane] : 0;
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += u;
    }
    if (lane < warps) scratch[lane] = inc - v;  // exclusive
    if (lane == 31) scratch[32] = inc;
  }
  __syncthreads();
  int result = scratch[warp] + in_warp;
  *total = scratch[32];
  __syncthreads();
  return result;
}

// Find the bucket holding the k-th smallest (1-based) of 256 counters: returns
// the bucket and the count of elements in lower buckets.  Warp 0 only; result
// through shared memory.
__device__ __forceinline__ void find_bucket(const uint32_t* hist, uint32_t k, uint32_t base,
                                            uint32_t* out_bucket, uint32_t* out_below) {
  const int lane = threadIdx.x & 31;
  uint32_t local[8], sum = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    local[j] = hist[lane * 8 + j];
    sum += local[j];
  }
  uint32_t inc = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t u = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += u;
  }
  uint32_t before = base + inc - sum;
  // the lane whose range [before, before+sum) contains the k-th element
  bool mine = before < k && k <= before + sum;
  if (mine) {
    uint32_t run = before;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (run < k && k <= run + local[j]) {
        *out_bucket = (uint32_t)(lane * 8 + j);
        *out_below = run;
      }
      run += local[j];
    }
  }
}

// Sort `count` composites (<= kSmemSort) held in shared memory ascending,
// padding to a power of two with UINT64_MAX.
__device__ void bitonic_sort(unsigned long long* data, int count) {
  int size = 32;
  while (size < count) size <<= 1;
  for (int i = count + threadIdx.x; i < size; i += blockDim.x) data[i] = ~0ull;
  __syncthreads();
  for (int span = 2; span <= size; span <<= 1) {
    for (int stride = span >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < size; i += blockDim.x) {
        int j = i ^ stride;
        if (j > i) {
          unsigned long long a = data[i], b = data[j];
          bool ascending = (i & span) == 0;
          if ((a > b) == ascending) {
            data[i] = b;
            data[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Ascending sort of n = E * blockDim.x 32-bit values in shared memory `data`
// (n a power of two; blockDim.x a power of two >= 32).  Thread t holds elements
// t*E .. t*E+E-1 in registers through the bitonic network: strides below E stay
// inside the thread, strides below 32*E are lane exchanges (shuffles), and only the
// larger strides go through shared memory (two barriers each).  For E = 2 and
// n = 512 that is 12 barriers instead of the 45 of a shared-memory network.
template <int E>
__device__ __forceinline__ void cmpx_in_thread(uint32_t (&v)[E], int s, int base, int span) {
#pragma unroll
  for (int ss = E / 2; ss >= 1; ss >>= 1) {
    if (ss != s) continue;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      if (e & ss) continue;
      const bool asc = ((base + e) & span) == 0;
      const uint32_t lo = min(v[e], v[e | ss]), hi = max(v[e], v[e | ss]);
      v[e] = asc ? lo : hi;
      v[e | ss] = asc ? hi : lo;
    }
  }
}

template <int E>
__device__ void block_sort_regs(uint32_t* data) {
  const int t = threadIdx.x, lane = t & 31, base = t * E;
  const int n = E * (int)blockDim.x;
  uint32_t v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = data[base + e];
  for (int span = 2; span <= n; span <<= 1) {
    for (int s = span >> 1; s > 0; s >>= 1) {
      if (s < E) {
        cmpx_in_thread<E>(v, s, base, span);
      } else if (s < 32 * E) {
        const int m = s / E;  // partner lane = lane ^ m; the lower lane keeps the minimum when ascending
        const bool low = (lane & m) == 0;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const uint32_t p = __shfl_xor_sync(0xffffffffu, v[e], m);
          const bool keep_min = low == (((base + e) & span) == 0);
          v[e] = keep_min ? min(v[e], p) : max(v[e], p);
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) data[base + e] = v[e];
        __syncthreads();
        const bool low = (base & s) == 0;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const uint32_t p = data[(base + e) ^ s];
          const bool keep_min = low == (((base + e) & span) == 0);
          v[e] = keep_min ? min(v[e], p) : max(v[e], p);
        }
        __syncthreads();
      }
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) data[base + e] = v[e];
  __syncthreads();
}

// block_sort_regs for a block of THREADS threads known at compile time: the whole
// network unrolled, so every stride and direction test is a constant.
template <int E, int THREADS>
__device__ void block_sort_fixed(uint32_t* data) {
  constexpr int LOGN = __builtin_ctz(E * THREADS);
  const int t = threadIdx.x, lane = t & 31, base = t * E;
  uint32_t v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = data[base + e];
#pragma unroll
  for (int ls = 1; ls <= LOGN; ++ls) {
    const int span = 1 << ls;
#pragma unroll
    for (int lt = ls - 1; lt >= 0; --lt) {
      const int s = 1 << lt;
      if (s < E) {
        cmpx_in_thread<E>(v, s, base, span);
      } else if (s < 32 * E) {
        const int m = s / E;
        const bool low = (lane & m) == 0;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const uint32_t p = __shfl_xor_sync(0xffffffffu, v[e], m);
          const bool keep_min = low == (((base + e) & span) == 0);
          v[e] = keep_min ? min(v[e], p) : max(v[e], p);
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) data[base + e] = v[e];
        __syncthreads();
        const bool low = (base & s) == 0;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const uint32_t p = data[(base + e) ^ s];
          const bool keep_min = low == (((base + e) & span) == 0);
          v[e] = keep_min ? min(v[e], p) : max(v[e], p);
        }
        __syncthreads();
      }
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) data[base + e] = v[e];
  __syncthreads();
}

template <int MAXE>
__device__ void block_sort_u32(uint32_t* data, int size);

// block_sort_u32 for blocks of exactly THREADS threads, with the unrolled networks.
template <int MAXE, int THREADS>
__device__ void block_sort_u32_fixed(uint32_t* data, int size) {
  if (size == THREADS) return block_sort_fixed<1, THREADS>(data);
  if (MAXE >= 2 && size == 2 * THREADS) return block_sort_fixed<(MAXE >= 2 ? 2 : 1), THREADS>(data);
  if (MAXE >= 4 && size == 4 * THREADS) return block_sort_fixed<(MAXE >= 4 ? 4 : 1), THREADS>(data);
  if (MAXE >= 8 && size == 8 * THREADS) return block_sort_fixed<(MAXE >= 8 ? 8 : 1), THREADS>(data);
  block_sort_u32<1>(data, size);  // shared-memory network (size below the block or above MAXE per thread)
}

// Ascending sort of `size` (a power of two >= 32) values in shared memory: the
// register network when size is a multiple of the block with E = size / blockDim.x
// up to MAXE (the caller's register budget), else a shared-memory bitonic network.
template <int MAXE>
__device__ void block_sort_u32(uint32_t* data, int size) {
  const int e = size / (int)blockDim.x;
  if (size >= (int)blockDim.x && e <= MAXE) {
    if (e == 1) return block_sort_regs<1>(data);
    if (MAXE >= 2 && e == 2) return block_sort_regs<(MAXE >= 2 ? 2 : 1)>(data);
    if (MAXE >= 4 && e == 4) return block_sort_regs<(MAXE >= 4 ? 4 : 1)>(data);
    if (MAXE >= 8 && e == 8) return block_sort_regs<(MAXE >= 8 ? 8 : 1)>(data);
  }
  for (int span = 2; span <= size; span <<= 1) {
    for (int stride = span >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < size; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const uint32_t a = data[i], c = data[j];
          if ((a > c) == ((i & span) == 0)) {
            data[i] = c;
            data[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Histogram increment with the warp's equal bins combined first (one shared-memory
// atomic per distinct bin per warp step); `live` lanes take part, all lanes call.
__device__ __forceinline__ void hist_add(uint32_t* hist, uint32_t bin, bool live) {
  const uint32_t mask = __ballot_sync(0xffffffffu, live);
  if (!live) return;
  const uint32_t peers = __match_any_sync(mask, bin);
  if ((threadIdx.x & 31) == (uint32_t)(__ffs(peers) - 1)) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
}

struct TopkArgs {
  KeySource src;
  int64_t n;        // keys per image
  int64_t k;        // winners per image
  bool nan_last;
  unsigned long long* sorted;  // [batch][sorted_pitch] composites (key<<32 | index)
  int64_t sorted_pitch;
  uint32_t* hist64k;           // [batch][65536] for the large-k path
  unsigned long long* scratch; // [batch][n] for the large-k path
};

__global__ void __launch_bounds__(kTopkThreads) topk_block(TopkArgs args) {
  __shared__ uint32_t hist[256];
  __shared__ int scan[33];
  __shared__ uint32_t sel_bucket, sel_below;
  __shared__ int collected;
  extern __shared__ unsigned long long cand[];
  const int64_t b = blockIdx.x;
  const int64_t n = args.n, k = args.k;
  unsigned long long* out = args.sorted + b * args.sorted_pitch;
  if (k <= 0) return;

  if (k > kSmemSort) {
    // Stable counting sort of all n keys (index order preserved within a key).
    uint32_t* h = args.hist64k + b * 65536;
    for (int i = threadIdx.x; i < 65536; i += blockDim.x) h[i] = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
      atomicAdd(&h[score_key(args.src.get(b, i), args.nan_last)], 1u);
    __syncthreads();
    // exclusive scan of 65536 counters: 64 per thread
    {
      uint32_t local = 0;
      const int per = 65536 / kTopkThreads;
      for (int j = 0; j < per; ++j) local += h[threadIdx.x * per + j];
      int dummy;
      // block scan of sums via the prefix helper on 32-bit values
      __shared__ uint32_t sums[kTopkThreads];
      sums[threadIdx.x] = local;
      __syncthreads();
      for (int o = 1; o < kTopkThreads; o <<= 1) {
        uint32_t add = threadIdx.x >= o ? sums[threadIdx.x - o] : 0u;
        __syncthreads();
        sums[threadIdx.x] += add;
        __syncthreads();
      }
      uint32_t run = sums[threadIdx.x] - local;
      for (int j = 0; j < per; ++j) {
        uint32_t c = h[threadIdx.x * per + j];
        h[threadIdx.x * per + j] = run;
        run += c;
      }
      (void)dummy;
    }
    __syncthreads();
    // ordered scatter by warp 0
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      for (int64_t base = 0; base < n; base += 32) {
        int64_t i = base + lane;
        bool valid = i < n;
        uint32_t key = valid ? score_key(args.src.get(b, i), args.nan_last) : 0xffffffffu;
        uint32_t peers = __match_any_sync(0xffffffffu, key);
        int rank = __popc(peers & lanemask_lt());
        int leader = __ffs(peers) - 1;
        uint32_t start = 0;
        if (lane == leader && valid) start = atomicAdd(&h[key], (uint32_t)__popc(peers));
        start = __shfl_sync(0xffffffffu, start, leader);
        if (valid) {
          uint32_t pos = start + rank;
          args.scratch[b * n + pos] = ((unsigned long long)key << 32) | (unsigned long long)i;
        }
        __syncwarp();
      }
    }
    __syncthreads();
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) out[i] = args.scratch[b * n + i];
    return;
  }

  // --- radix select of the k-th smallest 16-bit key
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
    atomicAdd(&hist[score_key(args.src.get(b, i), args.nan_last) >> 8], 1u);
  __syncthreads();
  if (threadIdx.x < 32) find_bucket(hist, (uint32_t)k, 0u, &sel_bucket, &sel_below);
  __syncthreads();
  const uint32_t high = sel_bucket, below_high = sel_below;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    uint32_t key = score_key(args.src.get(b, i), args.nan_last);
    if ((key >> 8) == high) atomicAdd(&hist[key & 255u], 1u);
  }
  __syncthreads();
  if (threadIdx.x < 32) find_bucket(hist, (uint32_t)k, below_high, &sel_bucket, &sel_below);
  __syncthreads();
  const uint32_t threshold = (high << 8) | sel_bucket;
  const int64_t need = k - (int64_t)sel_below;  // ties at the threshold to take, lowest index first

  // --- index-ordered collection
  if (threadIdx.x == 0) collected = 0;
  __syncthreads();
  int64_t eq_seen = 0;
  for (int64_t base = 0; base < n; base += blockDim.x) {
    int64_t i = base + threadIdx.x;
    uint32_t key = i < n ? score_key(args.src.get(b, i), args.nan_last) : 0xffffffffu;
    bool eq = key == threshold;
    int eq_total;
    int eq_rank = block_prefix(eq, scan, &eq_total);
    bool take = key < threshold || (eq && eq_seen + eq_rank < need);
    if (take) {
      int pos = atomicAdd(&collected, 1);
      cand[pos] = ((unsigned long long)key << 32) | (unsigned long long)i;
    }
    eq_seen += eq_total;
  }
  __syncthreads();
  bitonic_sort(cand, (int)k);
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) out[i] = cand[i];
}

// k <= 4096: 256-thread CTA per image (eight fit on an SM).
//  1. radix select of the k-th smallest 16-bit key (two 256-bin histograms);
//  2. index-ordered collection: warp w owns a contiguous index range, counts its
//     keys below / equal to the threshold with ballots, one block-wide prefix over
//     the 8 warp counts places every warp, then each warp writes its winners in
//     index order (the first `need` threshold ties globally);
//  3. the k winners sit in index order, so a sort by key alone is stable: bitonic
//     sort of (key << 12 | slot) 32-bit composites in shared memory.
constexpr int kSmallThreads = 256;
constexpr int kSmallWarps = kSmallThreads / 32;

constexpr int kStageKeys = 24576;  // keys staged in shared memory (48 KB)

// Top k of n 16-bit keys in one CTA of 32*WARPS threads: radix select of the
// k-th key, index-ordered collection of the winners, stable bitonic sort of
// (key << 12 | slot) composites.  comp and src are shared arrays of cap >= k
// (a power of two >= 32, k <= 4096); out[i] = key << 32 | index for i < k.
template <int WARPS, typename KeyAt>
__device__ void cta_topk(int n, int k, int cap, KeyAt key_at, uint32_t* comp, uint32_t* src,
                         unsigned long long* out) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel_bucket, sel_below;
  __shared__ int warp_lt[WARPS], warp_eq[WARPS];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int trips = (n + (int)blockDim.x - 1) / (int)blockDim.x;  // warp-uniform loop counts
  // --- radix select
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int r = 0; r < trips; ++r) {
    const int i = r * (int)blockDim.x + threadIdx.x;
    const bool live = i < n;
    hist_add(hist, live ? key_at(i) >> 8 : 0u, live);
  }
  __syncthreads();
  if (warp == 0) find_bucket(hist, (uint32_t)k, 0u, &sel_bucket, &sel_below);
  __syncthreads();
  const uint32_t high = sel_bucket, below_high = sel_below;
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int r = 0; r < trips; ++r) {
    const int i = r * (int)blockDim.x + threadIdx.x;
    const uint32_t key = i < n ? key_at(i) : 0xffffffffu;
    const bool live = (key >> 8) == high;
    hist_add(hist, key & 255u, live);
  }
  __syncthreads();
  if (warp == 0) find_bucket(hist, (uint32_t)k, below_high, &sel_bucket, &sel_below);
  __syncthreads();
  const uint32_t threshold = (high << 8) | sel_bucket;
  const int need = k - (int)sel_below;
  // --- index-ordered collection
  const int span = ((n + WARPS - 1) / WARPS + 31) / 32 * 32;
  const int lo = warp * span, hi = lo + span < n ? lo + span : n;
  int lt = 0, eq = 0;
  for (int base = lo; base < hi; base += 32) {
    const int i = base + lane;
    const uint32_t key = i < hi ? key_at(i) : 0xffffffffu;
    lt += __popc(__ballot_sync(0xffffffffu, key < threshold));
    eq += __popc(__ballot_sync(0xffffffffu, key == threshold));
  }
  if (lane == 0) {
    warp_lt[warp] = lt;
    warp_eq[warp] = eq;
  }
  __syncthreads();
  int eq_before = 0, taken_before = 0;
  for (int w = 0; w < warp; ++w) {
    int take_eq = need - eq_before;
    take_eq = take_eq < 0 ? 0 : (take_eq > warp_eq[w] ? warp_eq[w] : take_eq);
    taken_before += warp_lt[w] + take_eq;
    eq_before += warp_eq[w];
  }
  const uint32_t lane_lt = (1u << lane) - 1u;
  for (int base = lo; base < hi; base += 32) {
    const int i = base + lane;
    const uint32_t key = i < hi ? key_at(i) : 0xffffffffu;
    const uint32_t eq_mask = __ballot_sync(0xffffffffu, key == threshold);
    const int my_eq_rank = eq_before + __popc(eq_mask & lane_lt);
    const bool take = key < threshold || (key == threshold && my_eq_rank < need);
    const uint32_t take_mask = __ballot_sync(0xffffffffu, take);
    if (take) {
      const int pos = taken_before + __popc(take_mask & lane_lt);
      comp[pos] = (key << 12) | (uint32_t)pos;
      src[pos] = (uint32_t)i;
    }
    taken_before += __popc(take_mask);
    eq_before += __popc(eq_mask);
  }
  __syncthreads();
  // --- stable sort by key (slot order = index order)
  for (int i = k + threadIdx.x; i < cap; i += blockDim.x) comp[i] = 0xffffffffu;
  __syncthreads();
  block_sort_u32<4>(comp, cap);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const uint32_t c = comp[i];
    out[i] = ((unsigned long long)(c >> 12) << 32) | (unsigned long long)src[c & 0xfffu];
  }
}


template <bool kStaged>
__global__ void __launch_bounds__(kSmallThreads) topk_small(TopkArgs args) {
  extern __shared__ uint32_t dyn[];  // [cap] composites, [cap] source indices, [n] staged keys
  const int64_t b = blockIdx.x;
  const int n = (int)args.n, k = (int)args.k;
  int cap = 32;
  while (cap < k) cap <<= 1;
  uint32_t* comp = dyn;
  uint32_t* src = dyn + cap;
  uint16_t* staged = reinterpret_cast<uint16_t*>(dyn + 2 * cap);
  unsigned long long* out = args.sorted + b * args.sorted_pitch;
  if (k <= 0) return;
  const uint32_t* rec = args.src.records ? args.src.records + b * args.src.pitch : nullptr;
  const uint16_t* bits = args.src.records ? nullptr : args.src.bits + b * args.src.pitch;
  auto raw = [&](int i) -> uint16_t { return rec ? (uint16_t)(rec[i] & 0xffffu) : bits[i]; };
  if (kStaged) {  // one coalesced, 4-way unrolled pass computes every key once
    int i = threadIdx.x;
    for (; i + 3 * kSmallThreads < n; i += 4 * kSmallThreads) {
      const uint16_t h0 = raw(i), h1 = raw(i + kSmallThreads), h2 = raw(i + 2 * kSmallThreads),
                     h3 = raw(i + 3 * kSmallThreads);
      staged[i] = (uint16_t)score_key(h0, args.nan_last);
      staged[i + kSmallThreads] = (uint16_t)score_key(h1, args.nan_last);
      staged[i + 2 * kSmallThreads] = (uint16_t)score_key(h2, args.nan_last);
      staged[i + 3 * kSmallThreads] = (uint16_t)score_key(h3, args.nan_last);
    }
    for (; i < n; i += kSmallThreads) staged[i] = (uint16_t)score_key(raw(i), args.nan_last);
    __syncthreads();
  }
  auto key_at = [&](int i) -> uint32_t {
    return kStaged ? (uint32_t)staged[i] : score_key(raw(i), args.nan_last);
  };
  cta_topk<kSmallWarps>(n, k, cap, key_at, comp, src, out);
}

// Stage-1 top-k from the class max's per-image histogram of key high bytes
// (k <= 4096, anchors <= 65536): the bucket holding the k-th key comes from that
// histogram, so one pass over the records keeps only the candidates (high byte at
// or below that bucket) -- in index order, in a shared-memory segment per warp
// span -- and builds the low-byte histogram of the bucket; the threshold, the
// index-ordered collection and the sort then run on the candidates alone.  A CTA
// whose candidates overflow a segment falls back to the full top-k.
__host__ __device__ constexpr int hist_segment(int cap) { return cap / 4 > 512 ? cap / 4 : 512; }

// The top k of one image's records with the class max's high-byte histogram
// `key_hist` (256 counts).  `work` is shared memory of hist_topk_words(k) words;
// out[i] = key << 32 | anchor for i < k, in key order, ties in anchor order.
__host__ __device__ constexpr int topk_cap(int k) {
  int cap = 32;
  while (cap < k) cap <<= 1;
  return cap;
}
__host__ __device__ constexpr int hist_topk_words(int k) {
  return 2 * topk_cap(k) + kSmallWarps * hist_segment(topk_cap(k));
}

__device__ void hist_topk(const uint32_t* rec, int n, int k, bool nan_last, const uint32_t* key_hist,
                          uint32_t* work, unsigned long long* out) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel_bucket, sel_below;
  __shared__ int warp_lt[kSmallWarps], warp_eq[kSmallWarps];
  __shared__ int overflow;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cap = topk_cap(k);
  uint32_t* comp = work;
  uint32_t* src = work + cap;
  const int seg_cap = hist_segment(cap);
  uint32_t* seg = work + 2 * cap + warp * seg_cap;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = key_hist[i];
  if (threadIdx.x == 0) overflow = 0;
  __syncthreads();
  if (warp == 0) find_bucket(hist, (uint32_t)k, 0u, &sel_bucket, &sel_below);
  __syncthreads();
  const uint32_t high = sel_bucket, below_high = sel_below;
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  // one pass over the records: this warp's span of whole uint4 groups (n % 4 == 0),
  // four records per lane per load, candidates compacted in index order by a
  // warp scan of the per-lane counts
  const uint4* rec4 = reinterpret_cast<const uint4*>(rec);
  const int n4 = n >> 2;
  const int span4 = (n4 + kSmallWarps - 1) / kSmallWarps;
  const int lo4 = warp * span4, hi4 = lo4 + span4 < n4 ? lo4 + span4 : n4;
  const uint32_t lane_lt = (1u << lane) - 1u;
  int count = 0;
  constexpr int U = 4;  // uint4 loads in flight per lane
  for (int base = lo4; base < hi4; base += 32 * U) {
    uint4 q[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int g = base + u * 32 + lane;
      q[u] = g < hi4 ? __ldg(rec4 + g) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int g = base + u * 32 + lane;
      const uint32_t r4[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
      uint32_t key[4];
      int mine = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        key[j] = score_key((uint16_t)(r4[j] & 0xffffu), nan_last);
        mine += (g < hi4 && (key[j] >> 8) <= high) ? 1 : 0;
      }
      int incl = mine;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      int pos = count + incl - mine;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (g < hi4 && (key[j] >> 8) <= high) {
          if (pos < seg_cap) seg[pos] = (key[j] << 16) | (uint32_t)(4 * g + j);
          ++pos;
        }
      }
      count += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  if (lane == 0 && count > seg_cap) overflow = 1;
  __syncthreads();
  if (overflow) {  // candidates spill a segment (clustered scores): the full top-k, keys read again
    auto key_at = [&](int i) -> uint32_t { return score_key((uint16_t)(rec[i] & 0xffffu), nan_last); };
    cta_topk<kSmallWarps>(n, k, cap, key_at, comp, src, out);
    return;
  }
  // low bytes of the keys in the selected high-byte bucket, from the candidates
  for (int base = 0; base < count; base += 32) {
    const int j = base + lane;
    const uint32_t key = j < count ? seg[j] >> 16 : 0xffffffffu;
    hist_add(hist, key & 255u, (key >> 8) == high);
  }
  __syncthreads();
  if (warp == 0) find_bucket(hist, (uint32_t)k, below_high, &sel_bucket, &sel_below);
  __syncthreads();
  const uint32_t threshold = (high << 8) | sel_bucket;
  const int need = k - (int)sel_below;
  // index-ordered collection over the segments (warp order is index order)
  int lt = 0, eq = 0;
  for (int base = 0; base < count; base += 32) {
    const int j = base + lane;
    const uint32_t key = j < count ? seg[j] >> 16 : 0xffffffffu;
    lt += __popc(__ballot_sync(0xffffffffu, key < threshold));
    eq += __popc(__ballot_sync(0xffffffffu, key == threshold));
  }
  if (lane == 0) {
    warp_lt[warp] = lt;
    warp_eq[warp] = eq;
  }
  __syncthreads();
  int eq_before = 0, taken_before = 0;
  for (int w = 0; w < warp; ++w) {
    int take_eq = need - eq_before;
    take_eq = take_eq < 0 ? 0 : (take_eq > warp_eq[w] ? warp_eq[w] : take_eq);
    taken_before += warp_lt[w] + take_eq;
    eq_before += warp_eq[w];
  }
  for (int base = 0; base < count; base += 32) {
    const int j = base + lane;
    const uint32_t entry = j < count ? seg[j] : 0u;
    const uint32_t key = j < count ? entry >> 16 : 0xffffffffu;
    const uint32_t eq_mask = __ballot_sync(0xffffffffu, key == threshold);
    const int my_eq_rank = eq_before + __popc(eq_mask & lane_lt);
    const bool take = key < threshold || (key == threshold && my_eq_rank < need);
    const uint32_t take_mask = __ballot_sync(0xffffffffu, take);
    if (take) {
      const int pos = taken_before + __popc(take_mask & lane_lt);
      comp[pos] = (key << 12) | (uint32_t)pos;
      src[pos] = entry & 0xffffu;
    }
    taken_before += __popc(take_mask);
    eq_before += __popc(eq_mask);
  }
  __syncthreads();
  for (int i = k + threadIdx.x; i < cap; i += blockDim.x) comp[i] = 0xffffffffu;
  __syncthreads();
  block_sort_u32_fixed<4, kSmallThreads>(comp, cap);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const uint32_t c = comp[i];
    out[i] = ((unsigned long long)(c >> 12) << 32) | (unsigned long long)src[c & 0xfffu];
  }
}

__global__ void __launch_bounds__(kSmallThreads) topk_hist(TopkArgs args, const uint32_t* key_hist) {
  extern __shared__ uint32_t dyn[];
  const int64_t b = blockIdx.x;
  if (args.k <= 0) return;
  hist_topk(args.src.records + b * args.src.pitch, (int)args.n, (int)args.k, args.nan_last, key_hist + b * 256,
            dyn, args.sorted + b * args.sorted_pitch);
}

// --------------------------------------------------------- 3. pair gather

// pair_bits[b][r*nc + c] = score of class c at the stage-1 anchor of rank r.
__global__ void __launch_bounds__(256) gather_pairs(SelectView v, bool sigmoid,
                                                    const unsigned long long* stage1,
                                                    int64_t s1_pitch, int64_t k, uint16_t* pair_bits,
                                                    int64_t pair_pitch, uint16_t* trace_gathered) {
  const int64_t total = v.batch * k * v.classes;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    int64_t b = t / (k * v.classes), flat = t % (k * v.classes);
    int64_t r = flat / v.classes, c = flat % v.classes;
    int64_t anchor = (int64_t)(stage1[b * s1_pitch + r] & 0xffffffffull);
    uint16_t bits = score_bits(v, b, anchor, c, sigmoid);
    pair_bits[b * pair_pitch + flat] = bits;
    if (trace_gathered) trace_gathered[t] = bits;
  }
}

// ------------------------------------- 3'. fused pair stage and pack

// Class-aware stage 2 and pack for one image per CTA, without gathering the
// k x nc scores.  K1 = the k-th stage-1 key.  The k pairs (rank r, best class of
// anchor r) all have keys <= K1, so every pair of the final top k has a key
// <= K1 too; a non-best class of anchor r can qualify only if the best score
// among its other classes has key <= K1 (the class-max pass records that key,
// from the second-largest logit, or from the exact rescan for the anchors it
// rescans).  Candidates: (r, best class) for every other
// anchor, and every class with key <= K1 of the anchors that may hold more
// (read exactly, as gather_pairs does).  Up to kPairCand candidates, as 32-bit
// composites (key << 15 | r*nc + c), are sorted ascending in shared memory --
// equal keys in flat-index order, as the stage-2 top-k orders them -- and the
// first k packed.  More candidates (many ties at K1) take the exact top-k over
// all k*nc pairs in the same CTA, keys read on the fly.
constexpr int kPairThreads = 256;
constexpr int kPairCand = 4096;
constexpr int64_t kPairFlatMax = 1 << 15;

__global__ void __launch_bounds__(kPairThreads) pairs_fused(SelectView v, bool nan_last, bool sigmoid, int k,
                                                            const unsigned long long* stage1, int64_t s1_pitch,
                                                            const uint32_t* records, const uint16_t* second_keys,
                                                            float* out) {
  // [kPairCand] composites (reused as k sorted 64-bit results on overflow),
  // [k] ranks of anchors needing every class, [2 * cap] top-k scratch
  extern __shared__ uint32_t pair_cand[];
  __shared__ int count, n_full;
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nc = (int)v.classes;
  int cap = 32;
  while (cap < k) cap <<= 1;
  int* full = reinterpret_cast<int*>(pair_cand + kPairCand);
  uint32_t* topk_comp = pair_cand + kPairCand + k;
  const unsigned long long* s1 = stage1 + (int64_t)b * s1_pitch;
  const uint32_t k1 = (uint32_t)(s1[k - 1] >> 32);
  if (tid == 0) count = n_full = 0;
  __syncthreads();
  for (int r = tid; r < k; r += kPairThreads) {
    const unsigned long long e = s1[r];
    const int64_t a = (int64_t)(e & 0xffffffffull);
    if ((uint32_t)second_keys[(int64_t)b * v.anchors + a] > k1) {  // only the best class can rank
      const uint32_t cls = records[(int64_t)b * v.anchors + a] >> 16;
      const int slot = atomicAdd(&count, 1);
      if (slot < kPairCand) pair_cand[slot] = ((uint32_t)(e >> 32) << 15) | (uint32_t)(r * nc + (int)cls);
    } else {
      full[atomicAdd(&n_full, 1)] = r;
    }
  }
  __syncthreads();
  for (int f = warp; f < n_full; f += kPairThreads / 32) {  // warp per anchor, lanes over classes
    const int r = full[f];
    const int64_t a = (int64_t)(s1[r] & 0xffffffffull);
    for (int c = lane; c < nc; c += 32) {
      const uint32_t key = score_key(score_bits(v, b, a, c, sigmoid), nan_last);
      if (key <= k1) {
        const int slot = atomicAdd(&count, 1);
        if (slot < kPairCand) pair_cand[slot] = (key << 15) | (uint32_t)(r * nc + c);
      }
    }
  }
  __syncthreads();
  const int n = count;  // >= k: the k best-class pairs are always candidates
  auto pack = [&](int j, int flat) {
    const int r = flat / nc, c = flat - r * nc;
    const int64_t anchor = (int64_t)(s1[r] & 0xffffffffull);
    const uint16_t bits = score_bits(v, b, anchor, c, sigmoid);
    const uint16_t* box = v.base + (int64_t)b * v.sb + anchor * v.sa;
    const int64_t t = (int64_t)b * k + j;
    uint32_t* row = reinterpret_cast<uint32_t*>(out + t * 6);
#pragma unroll
    for (int q = 0; q < 4; ++q) row[q] = float_bits_of_half(box[q * v.sc]);
    row[4] = float_bits_of_half(bits);
    out[t * 6 + 5] = (float)c;
  };
  if (n > kPairCand) {
    unsigned long long* sorted = reinterpret_cast<unsigned long long*>(pair_cand);
    auto key_at = [&](int i) -> uint32_t {
      const int r = i / nc, c = i - r * nc;
      return score_key(score_bits(v, b, (int64_t)(s1[r] & 0xffffffffull), c, sigmoid), nan_last);
    };
    cta_topk<kPairThreads / 32>(k * nc, k, cap, key_at, topk_comp, topk_comp + cap, sorted);
    __syncthreads();
    for (int j = tid; j < k; j += kPairThreads) pack(j, (int)(sorted[j] & 0xffffffffull));
    return;
  }
  int size = 32;
  while (size < n) size <<= 1;
  for (int i = n + tid; i < size; i += kPairThreads) pair_cand[i] = 0xffffffffu;
  __syncthreads();
  block_sort_u32<8>(pair_cand, size);
  for (int j = tid; j < k; j += kPairThreads) pack(j, (int)(pair_cand[j] & 0x7fffu));
}

// Stage 1, the class-aware pair stage and the pack for one image per CTA
// (planar sigmoid scores, k <= 2048, no trace).  The stage-1 top-k (hist_topk)
// stays in shared memory; right after it each of the k anchors' record, second
// key and four box values are read in one batch, so the pack touches global
// memory only for the rare non-best classes of anchors gathered in full.  The
// candidate rule and ordering are those of pairs_fused.
// Shared memory in words: stage-1 (2k), boxes (2k), records (k), then the
// top-k work area, reused by the pair candidates.
__host__ __device__ constexpr int finish_work_offset(int k) { return (5 * k + 1) & ~1; }
__host__ __device__ constexpr int finish_words(int k) {
  return finish_work_offset(k) + (hist_topk_words(k) > kPairCand + k + 2 * topk_cap(k)
                                      ? hist_topk_words(k)
                                      : kPairCand + k + 2 * topk_cap(k));
}

__global__ void __launch_bounds__(kSmallThreads) select_finish(SelectView v, bool nan_last, int k,
                                                               const uint32_t* records,
                                                               const uint16_t* second_keys,
                                                               const uint32_t* key_hist, float* out) {
  extern __shared__ __align__(16) unsigned long long finish_smem[];
  __shared__ int count, n_full;
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const int nc = (int)v.classes;
  uint32_t* words = reinterpret_cast<uint32_t*>(finish_smem);
  unsigned long long* s1 = finish_smem;
  uint2* boxes = reinterpret_cast<uint2*>(words + 2 * k);
  uint32_t* recs = words + 4 * k;
  uint32_t* work = words + finish_work_offset(k);
  const uint32_t* rec_b = records + (int64_t)b * v.anchors;
  const uint16_t* box_b = v.base + (int64_t)b * v.sb;  // planar: anchor stride 1
  hist_topk(rec_b, (int)v.anchors, k, nan_last, key_hist + (int64_t)b * 256, work, s1);
  if (tid == 0) count = n_full = 0;
  __syncthreads();
  const uint32_t k1 = (uint32_t)(s1[k - 1] >> 32);
  uint32_t* pair_cand = work;
  int* full = reinterpret_cast<int*>(work + kPairCand);
  uint32_t* topk_comp = work + kPairCand + k;
  const uint32_t lane_lt = (1u << lane) - 1u;
  // appends to a shared list with one atomic per warp
  auto append = [&](int* counter, bool take) -> int {
    const uint32_t m = __ballot_sync(0xffffffffu, take);
    int first = 0;
    if (lane == 0 && m) first = atomicAdd(counter, __popc(m));
    return __shfl_sync(0xffffffffu, first, 0) + __popc(m & lane_lt);
  };
  for (int base = 0; base < k; base += kSmallThreads) {  // CTA-uniform trips for the ballots
    const int r = base + tid;
    const bool live = r < k;
    const unsigned long long e = live ? s1[r] : 0ull;
    const int a = (int)(e & 0xffffffffull);
    uint32_t rec = 0, second = 0xffffffffu, q[4] = {0u, 0u, 0u, 0u};
    if (live) {
      rec = rec_b[a];
      second = second_keys[(int64_t)b * v.anchors + a];
#pragma unroll
      for (int j = 0; j < 4; ++j) q[j] = box_b[a + j * v.sc];
      recs[r] = rec;
      boxes[r] = make_uint2(q[0] | (q[1] << 16), q[2] | (q[3] << 16));
    }
    const bool best_only = live && second > k1;  // only the best class can rank
    const int slot = append(&count, best_only);
    if (best_only && slot < kPairCand)
      pair_cand[slot] = ((uint32_t)(e >> 32) << 15) | (uint32_t)(r * nc + (int)(rec >> 16));
    const int fslot = append(&n_full, live && !best_only);
    if (live && !best_only) full[fslot] = r;
  }
  __syncthreads();
  // every class of the anchors that may hold more than their best: (anchor, class)
  // items over the whole CTA, four score loads in flight per thread
  const int items = n_full * nc;
  for (int base = 0; base < items; base += 4 * kSmallThreads) {
    uint16_t raw[4];
    int flat[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = base + u * kSmallThreads + tid;
      flat[u] = -1;
      raw[u] = 0;
      if (t < items) {
        const int f = t / nc, c = t - f * nc;
        const int r = full[f];
        raw[u] = box_b[(int64_t)(s1[r] & 0xffffffffull) + (int64_t)(c + 4) * v.sc];
        flat[u] = r * nc + c;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t key = flat[u] >= 0 ? score_key(sigmoid_h_fast(raw[u]), nan_last) : 0xffffffffu;
      const bool take = flat[u] >= 0 && key <= k1;
      const int slot = append(&count, take);
      if (take && slot < kPairCand) pair_cand[slot] = (key << 15) | (uint32_t)flat[u];
    }
  }
  __syncthreads();
  const int n = count;  // >= k: the k best-class pairs are always candidates
  auto pack = [&](int j, int flat) {
    const int r = flat / nc, c = flat - r * nc;
    const uint32_t rec = recs[r];
    const uint16_t bits = c == (int)(rec >> 16) ? (uint16_t)(rec & 0xffffu)
                                                 : score_bits(v, b, (int64_t)(s1[r] & 0xffffffffull), c, true);
    const uint2 bx = boxes[r];
    const int64_t t = (int64_t)b * k + j;
    uint32_t* row = reinterpret_cast<uint32_t*>(out + t * 6);
    row[0] = float_bits_of_half((uint16_t)(bx.x & 0xffffu));
    row[1] = float_bits_of_half((uint16_t)(bx.x >> 16));
    row[2] = float_bits_of_half((uint16_t)(bx.y & 0xffffu));
    row[3] = float_bits_of_half((uint16_t)(bx.y >> 16));
    row[4] = float_bits_of_half(bits);
    out[t * 6 + 5] = (float)c;
  };
  if (n > kPairCand) {  // many ties at K1: the exact top-k over all k*nc pairs, keys read on the fly
    unsigned long long* sorted = reinterpret_cast<unsigned long long*>(pair_cand);
    auto key_at = [&](int i) -> uint32_t {
      const int r = i / nc, c = i - r * nc;
      return score_key(score_bits(v, b, (int64_t)(s1[r] & 0xffffffffull), c, true), nan_last);
    };
    cta_topk<kSmallWarps>(k * nc, k, topk_cap(k), key_at, topk_comp, topk_comp + topk_cap(k), sorted);
    __syncthreads();
    for (int j = tid; j < k; j += kSmallThreads) pack(j, (int)(sorted[j] & 0xffffffffull));
    return;
  }
  int size = 32;
  while (size < n) size <<= 1;
  for (int i = n + tid; i < size; i += kSmallThreads) pair_cand[i] = 0xffffffffu;
  __syncthreads();
  block_sort_u32_fixed<8, kSmallThreads>(pair_cand, size);
  for (int j = tid; j < k; j += kSmallThreads) pack(j, (int)(pair_cand[j] & 0x7fffu));
}

// ------------------------------------------------------------------ 4. pack

struct PackArgs {
  SelectView v;
  bool agnostic;
  int64_t k;
  const uint32_t* records;
  int64_t rec_pitch;
  const unsigned long long* stage1;
  int64_t s1_pitch;
  const unsigned long long* stage2;
  int64_t s2_pitch;
  const uint16_t* pair_bits;
  int64_t pair_pitch;
  float* out;
  ttn_select_trace trace;
};

__global__ void __launch_bounds__(256) pack_rows(PackArgs p) {
  const int64_t total = p.v.batch * p.k;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    int64_t b = t / p.k, j = t % p.k;
    int64_t anchor, cls, flat = 0;
    uint32_t bits;
    int64_t first = (int64_t)(p.stage1[b * p.s1_pitch + j] & 0xffffffffull);
    if (p.agnostic) {
      anchor = first;
      uint32_t rec = p.records[b * p.rec_pitch + anchor];
      bits = rec & 0xffffu;
      cls = rec >> 16;
    } else {
      flat = (int64_t)(p.stage2[b * p.s2_pitch + j] & 0xffffffffull);
      int64_t rank = flat / p.v.classes;
      cls = flat % p.v.classes;
      anchor = (int64_t)(p.stage1[b * p.s1_pitch + rank] & 0xffffffffull);
      bits = p.pair_bits[b * p.pair_pitch + flat];
    }
    const uint16_t* box = p.v.base + b * p.v.sb + anchor * p.v.sa;
    uint32_t* row = reinterpret_cast<uint32_t*>(p.out + t * 6);
#pragma unroll
    for (int c = 0; c < 4; ++c) row[c] = float_bits_of_half(box[c * p.v.sc]);
    row[4] = float_bits_of_half(bits);
    p.out[t * 6 + 5] = (float)cls;
    if (p.trace.stage1_indices) p.trace.stage1_indices[t] = first;
    if (p.trace.top_values) p.trace.top_values[t] = (uint16_t)bits;
    if (p.trace.stage2_indices && !p.agnostic) p.trace.stage2_indices[t] = flat;
    if (p.trace.anchor_indices) p.trace.anchor_indices[t] = anchor;
    if (p.trace.labels) p.trace.labels[t] = cls;
  }
}

// --------------------------------------------------------------- host side

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct Workspace {
  size_t records, second, key_hist, stage1, pairs, stage2, hist, scratch, total;
};

ttn_status launch_topk(const TopkArgs& args, int64_t batch, int64_t k, cudaStream_t s) {
  if (k > kSmemSort) {
    topk_block<<<(unsigned)batch, kTopkThreads, 32 * 8, s>>>(args);
    return launch_check("ttn_select_f16 topk (large k)");
  }
  int cap = 32;
  while (cap < k) cap <<= 1;
  if (args.n <= kStageKeys) {
    const size_t smem = (size_t)cap * 8 + (size_t)(args.n + 1) / 2 * 4;  // + 16-bit staged keys
    TTN_TRY(ensure_dynamic_smem((const void*)topk_small<true>, (int)smem));
    topk_small<true><<<(unsigned)batch, kSmallThreads, smem, s>>>(args);
  } else {
    const size_t smem = (size_t)cap * 8;  // composites + source indices
    TTN_TRY(ensure_dynamic_smem((const void*)topk_small<false>, (int)smem));
    topk_small<false><<<(unsigned)batch, kSmallThreads, smem, s>>>(args);
  }
  return launch_check("ttn_select_f16 topk");
}

Workspace layout(int64_t batch, int64_t anchors, int64_t classes, int64_t k, bool agnostic) {
  Workspace w;
  int64_t kp = k < 1 ? 1 : k;
  int64_t pairs = agnostic ? 0 : kp * classes;
  w.records = 0;
  size_t off = align256((size_t)batch * anchors * 4);
  w.second = off;
  off += agnostic ? 0 : align256((size_t)batch * anchors * 2);
  w.key_hist = off;
  off += align256((size_t)batch * 256 * 4);
  w.stage1 = off;
  off += align256((size_t)batch * kp * 8);
  w.pairs = off;
  off += align256((size_t)batch * pairs * 2);
  w.stage2 = off;
  off += align256((size_t)batch * kp * 8);
  w.hist = off;
  bool large = k > kSmemSort;
  off += large ? align256((size_t)batch * 65536 * 4) : 0;
  w.scratch = off;
  int64_t widest = anchors > pairs ? anchors : pairs;
  off += large ? align256((size_t)batch * widest * 8) : 0;
  w.total = off;
  return w;
}

}  // namespace
}  // namespace ttn

using namespace ttn;

extern "C" {

size_t ttn_select_workspace_size(int64_t batch, int64_t anchors, int64_t classes, int64_t max_det,
                                 uint32_t flags) {
  if (batch <= 0 || anchors <= 0 || classes <= 0) return 256;
  int64_t k = max_det < anchors ? max_det : anchors;
  if (k < 0) k = 0;
  return layout(batch, anchors, classes, k, (flags & TTN_SELECT_AGNOSTIC) != 0).total;
}

ttn_status ttn_select_f16(const ttn_tensor* decoded, int64_t max_det, uint32_t flags,
                          void* workspace, size_t workspace_bytes, float* out,
                          const ttn_select_trace* trace, ttn_stream stream) {
  const char* name = "ttn_select_f16";
  TTN_TRY(validate(decoded, name));
  if (decoded->dtype != TTN_F16 || decoded->ndim != 3)
    return fail(TTN_INVALID_ARG, "%s: detection_select expects FP16 [B,A,4+nc]", name);
  if (decoded->sizes[2] <= 4 || max_det < 0)
    return fail(TTN_INVALID_ARG, "%s: detection_select requires nc > 0 and max_det >= 0", name);
  if (flags & ~(uint32_t)(TTN_SELECT_AGNOSTIC | TTN_SELECT_NAN_LAST | TTN_SELECT_SIGMOID))
    return fail(TTN_INVALID_ARG, "%s: unknown flag bits", name);
  SelectView v;
  v.base = (const uint16_t*)decoded->data;
  v.sb = decoded->strides[0];
  v.sa = decoded->strides[1];
  v.sc = decoded->strides[2];
  v.batch = decoded->sizes[0];
  v.anchors = decoded->sizes[1];
  v.classes = decoded->sizes[2] - 4;
  if (v.classes > 65535) return fail(TTN_UNSUPPORTED, "%s: more than 65535 classes", name);
  if (v.anchors > 0x7fffffffLL) return fail(TTN_UNSUPPORTED, "%s: too many anchors", name);
  const bool agnostic = flags & TTN_SELECT_AGNOSTIC, nan_last = flags & TTN_SELECT_NAN_LAST;
  const bool sigmoid = flags & TTN_SELECT_SIGMOID;
  const int64_t k = max_det < v.anchors ? max_det : v.anchors;
  if (!v.batch || !v.anchors) return TTN_OK;
  if (!agnostic && k * v.classes > 0x7fffffffLL)
    return fail(TTN_UNSUPPORTED, "%s: k*nc exceeds 2^31", name);
  Workspace w = layout(v.batch, v.anchors, v.classes, k, agnostic);
  if (!workspace || workspace_bytes < w.total || ((uintptr_t)workspace & 255u))
    return fail(TTN_INVALID_ARG, "%s: workspace needs %zu bytes, 256-byte aligned", name, w.total);
  if (k && !out) return fail(TTN_INVALID_ARG, "%s: null output", name);
  ttn_select_trace tr = trace ? *trace : ttn_select_trace{};
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = (uint8_t*)workspace;
  uint32_t* records = (uint32_t*)(ws + w.records);
  unsigned long long* stage1 = (unsigned long long*)(ws + w.stage1);
  uint16_t* pairs = (uint16_t*)(ws + w.pairs);
  unsigned long long* stage2 = (unsigned long long*)(ws + w.stage2);
  uint32_t* hist = (uint32_t*)(ws + w.hist);
  unsigned long long* scratch = (unsigned long long*)(ws + w.scratch);
  const int64_t kp = k < 1 ? 1 : k;

  // 1. class max
  bool planar = v.sa == 1 && v.anchors % 8 == 0 && v.sb % 8 == 0 && v.sc % 8 == 0 &&
                ((uintptr_t)(v.base + 4 * v.sc) & 15u) == 0;
  const bool traced = tr.class_max || tr.stage1_indices || tr.gathered_scores || tr.stage2_indices ||
                      tr.top_values || tr.anchor_indices || tr.labels;
  int pair_cap = 32;
  while (pair_cap < k && pair_cap < 4096) pair_cap <<= 1;
  const size_t pair_smem = (size_t)kPairCand * 4 + (size_t)k * 4 + (size_t)pair_cap * 8;
  // k <= 2048: the overflow path's k 64-bit results fit the candidate array
  const bool fused = planar && sigmoid && !agnostic && !traced && k >= 1 && k <= 2048 &&
                     k * v.classes <= kPairFlatMax && (int64_t)pair_smem <= max_dynamic_smem();
  uint16_t* second = fused ? (uint16_t*)(ws + w.second) : nullptr;
  // the stage-1 top-k from a histogram the class max builds (planar sigmoid path)
  const bool from_hist = planar && sigmoid && k >= 1 && k <= kSmemSort && v.anchors <= 65536;
  uint32_t* key_hist = from_hist ? (uint32_t*)(ws + w.key_hist) : nullptr;
  if (from_hist)
    TTN_TRY(cuda_check(cudaMemsetAsync(key_hist, 0, (size_t)v.batch * 256 * 4, s), "ttn_select_f16 memset"));
  if (planar && sigmoid) {
    int64_t work = v.batch * (v.anchors / 4);
    class_max_planar_sigmoid<4><<<grid_for(work, 256, 8), 256, 0, s>>>(v, nan_last, records, v.anchors,
                                                                       tr.class_max, second, key_hist);
  } else if (planar) {
    int64_t work = v.batch * (v.anchors / 8);
    class_max_planar8<<<grid_for(work, 256, 8), 256, 0, s>>>(v, nan_last, sigmoid, records,
                                                             v.anchors, tr.class_max);
  } else if (v.sc == 1 && v.classes >= 16) {
    int64_t work = v.batch * v.anchors * 32;
    class_max_warp<<<grid_for(work, 256, 8), 256, 0, s>>>(v, nan_last, sigmoid, records, v.anchors,
                                                          tr.class_max);
  } else {
    int64_t work = v.batch * v.anchors;
    class_max_thread<<<grid_for(work, 256, 8), 256, 0, s>>>(v, nan_last, sigmoid, records,
                                                            v.anchors, tr.class_max);
  }
  TTN_TRY(launch_check("ttn_select_f16 class_max"));
  if (!k) return TTN_OK;

  // 2'-3'. class-aware without trace from the histogram: top-k, pairs and pack in one kernel
  if (fused && from_hist && finish_words((int)k) * 4 <= max_dynamic_smem()) {
    const int smem = finish_words((int)k) * 4;
    TTN_TRY(ensure_dynamic_smem((const void*)select_finish, smem));
    select_finish<<<(unsigned)v.batch, kSmallThreads, smem, s>>>(v, nan_last, (int)k, records, second, key_hist,
                                                                 out);
    return launch_check("ttn_select_f16 finish");
  }

  // 2. stage-1 top-k over anchors
  TopkArgs t1{KeySource{records, nullptr, v.anchors}, v.anchors, k, nan_last, stage1, kp, hist, scratch};
  if (from_hist) {
    const size_t smem = (size_t)hist_topk_words((int)k) * 4;
    TTN_TRY(ensure_dynamic_smem((const void*)topk_hist, (int)smem));
    topk_hist<<<(unsigned)v.batch, kSmallThreads, smem, s>>>(t1, key_hist);
    TTN_TRY(launch_check("ttn_select_f16 topk"));
  } else {
    TTN_TRY(launch_topk(t1, v.batch, k, s));
  }

  // 3'. class-aware without trace: candidate pairs, sort and pack in one kernel
  if (fused) {
    TTN_TRY(ensure_dynamic_smem((const void*)pairs_fused, (int)pair_smem));
    pairs_fused<<<(unsigned)v.batch, kPairThreads, pair_smem, s>>>(v, nan_last, sigmoid, (int)k, stage1, kp,
                                                                   records, second, out);
    return launch_check("ttn_select_f16 pairs");
  }

  // 3. class-aware: pairs and stage-2 top-k
  if (!agnostic) {
    int64_t work = v.batch * k * v.classes;
    gather_pairs<<<grid_for(work, 256, 8), 256, 0, s>>>(v, sigmoid, stage1, kp, k, pairs,
                                                        kp * v.classes, tr.gathered_scores);
    TTN_TRY(launch_check("ttn_select_f16 gather_pairs"));
    TopkArgs t2{KeySource{nullptr, pairs, kp * v.classes}, k * v.classes, k, nan_last, stage2, kp,
                hist, scratch};
    TTN_TRY(launch_topk(t2, v.batch, k, s));
  }

  // 4. pack
  PackArgs p{v, agnostic, k, records, v.anchors, stage1, kp, stage2, kp, pairs, kp * v.classes, out, tr};
  pack_rows<<<grid_for(v.batch * k, 256, 8), 256, 0, s>>>(p);
  return launch_check("ttn_select_f16 pack");
}

}  // extern "C"
