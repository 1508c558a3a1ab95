// Softmax over any dim of a strided view (attention rows, DFL bins) and the
// fused Detect decode (DFL softmax + expectation + anchor decode + sigmoid).
//
// Softmax follows CPU eager's three IEEE passes: m = max (NaN-propagating),
// s = sum exp(x - m), y = exp(x - m) * (1/s), all in FP32 with one rounding of
// y.  So rows holding NaN, +inf or only -inf become NaN exactly as on CPU.
// Rows with a unit-stride reduction run one warp per row (values held in
// registers, 16-byte loads when rows are 8-aligned); reductions over a strided
// dim run one thread per row with consecutive threads on the unit-stride dim,
// which keeps every pass coalesced.
#include "common.cuh"

namespace ttn {
namespace {

__device__ __forceinline__ float nan_max(float a, float b) { return (b > a || b != b) ? b : a; }

// Row max for softmax.  A plain max is enough: a NaN anywhere in the row, an
// +inf (inf - inf), or an all -inf row (-inf - -inf) makes the sum NaN, so the
// whole row comes out NaN exactly as CPU eager's three passes produce.
__device__ __forceinline__ float row_max(float a, float b) { return fmaxf(a, b); }

// exp(v - m') as ex2 of one FMA, v*log2e - hi with hi = fl(m*log2e): the shift
// m' = hi/log2e differs from m by at most one rounding of m*log2e, and a shift
// common to a whole row cancels in the softmax ratio, so only the FMA's own
// rounding (2^-24 of the argument) reaches the probabilities.  The row maximum
// still maps to an argument within that rounding of 0, so nothing overflows.
struct ShiftLog2 {
  float hi;
};
__device__ __forceinline__ ShiftLog2 shift_log2(float m) { return {m * 1.44269504088896341f}; }
__device__ __forceinline__ float exp_shifted(float v, ShiftLog2 ml) {
  return ex2_approx(__fmaf_rn(v, 1.44269504088896341f, -ml.hi));
}

template <typename T>
__device__ __forceinline__ float load_scaled(const T* p, int64_t off, float scale, bool scaled) {
  if constexpr (sizeof(T) == 2) {
    float v = __half2float(reinterpret_cast<const __half*>(p)[off]);
    return scaled ? __half2float(__float2half_rn(__fmul_rn(v, scale))) : v;
  } else {
    float v = p[off];
    return scaled ? __fmul_rn(v, scale) : v;
  }
}

template <typename U>
__device__ __forceinline__ void store_out(U* p, int64_t off, float v) {
  if constexpr (sizeof(U) == 2) reinterpret_cast<__half*>(p)[off] = __float2half_rn(v);
  else p[off] = v;
}

struct RowSpace {  // non-reduced dims (innermost first) with x and y strides
  int ndim;
  int64_t size[7];
  int64_t sx[7];
  int64_t sy[7];
};

__device__ __forceinline__ void row_offsets(const RowSpace& rs, int64_t row, int64_t& ox,
                                            int64_t& oy) {
  ox = oy = 0;
#pragma unroll
  for (int d = 0; d < 7; ++d) {
    if (d >= rs.ndim) break;
    int64_t q = row / rs.size[d];
    int64_t r = row - q * rs.size[d];
    row = q;
    ox += r * rs.sx[d];
    oy += r * rs.sy[d];
  }
}

// One warp per row, unit-stride reduction, up to 32*PER elements per row.
template <typename T, typename U, int PER>
__global__ void __launch_bounds__(256) softmax_warp_rows(const T* x, U* y, RowSpace rs, int64_t rows,
                                                         int reduce, float scale, bool scaled) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = warp; row < rows; row += warps) {
    int64_t ox, oy;
    row_offsets(rs, row, ox, oy);
    float v[PER];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int e = k * 32 + lane;
      v[k] = e < reduce ? load_scaled(x, ox + e, scale, scaled) : -INFINITY;
      if (e < reduce) m = nan_max(m, v[k]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = nan_max(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int e = k * 32 + lane;
      if (e < reduce) {
        v[k] = exp_fast(__fsub_rn(v[k], m));
        s = __fadd_rn(s, v[k]);
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    const float inv = __fdiv_rn(1.0f, s);
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int e = k * 32 + lane;
      if (e < reduce) store_out(y, oy + e, __fmul_rn(v[k], inv));
    }
  }
}

// fp16 rows with reduce % 8 == 0 and 16-byte aligned rows: each lane owns whole
// 8-element vectors (element index (k*32 + lane)*8 + j).
template <int PER>
__global__ void __launch_bounds__(256) softmax_warp_rows_h8(const uint16_t* x, uint16_t* y, RowSpace rs,
                                                            int64_t rows, int reduce, float scale,
                                                            bool scaled) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int nvec = reduce >> 3;
  for (int64_t row = warp; row < rows; row += warps) {
    int64_t ox, oy;
    row_offsets(rs, row, ox, oy);
    const uint4* xv = reinterpret_cast<const uint4*>(x + ox);
    uint4* yv = reinterpret_cast<uint4*>(y + oy);
    float v[PER][8];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int e = k * 32 + lane;
      if (e < nvec) {
        uint4 q = xv[e];
        uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = __half22float2(*reinterpret_cast<__half2*>(&w[j]));
          if (scaled) {
            f.x = __half2float(__float2half_rn(__fmul_rn(f.x, scale)));
            f.y = __half2float(__float2half_rn(__fmul_rn(f.y, scale)));
          }
          v[k][2 * j] = f.x;
          v[k][2 * j + 1] = f.y;
          m = row_max(row_max(m, f.x), f.y);
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = row_max(m, __shfl_xor_sync(0xffffffffu, m, o));
    const ShiftLog2 ml = shift_log2(m);
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int e = k * 32 + lane;
      if (e < nvec) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[k][j] = exp_shifted(v[k][j], ml);
          s = __fadd_rn(s, v[k][j]);
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    const float inv = __fdiv_rn(1.0f, s);
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int e = k * 32 + lane;
      if (e < nvec) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          __half2 h = __floats2half2_rn(__fmul_rn(v[k][2 * j], inv), __fmul_rn(v[k][2 * j + 1], inv));
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        yv[e] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

// Contiguous fp16 rows (row pitch == reduce, 16-byte aligned, reduce % 8 == 0,
// reduce <= 1024): each warp streams its rows through a ring of SLOTS row buffers
// in shared memory with cp.async 16-byte copies, so SLOTS - 1 rows are in flight
// while the current one is reduced; completion is tracked by cp.async.wait_group
// (no software spin).  Rows of up to 512 fp16 take four slots (three rows of
// 1 KB or less in flight per warp keep enough bytes moving at small batches),
// longer rows two.
constexpr int kRowsWarps = 8;
constexpr int kRowMaxVec = 128;  // 1024 fp16 per row

template <int PER, int SLOTS>
__global__ void __launch_bounds__(kRowsWarps * 32) softmax_rows_pipelined(const uint16_t* x, uint16_t* y,
                                                                          int64_t rows, int reduce,
                                                                          float scale, bool scaled) {
  extern __shared__ __align__(16) uint4 rowbuf[];  // [warps][SLOTS][nvec]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = reduce >> 3;
  uint4* buf = rowbuf + (size_t)warp * SLOTS * nvec;
  const int64_t warps = (int64_t)gridDim.x * kRowsWarps;
  int64_t row = (int64_t)blockIdx.x * kRowsWarps + warp;
  auto prefetch = [&](int64_t r, int slot) {
    if (r < rows) {
      const uint4* src = reinterpret_cast<const uint4*>(x + r * reduce);
      for (int e = lane; e < nvec; e += 32) cp_async16(&buf[slot * nvec + e], &src[e]);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int k = 0; k < SLOTS - 1; ++k) prefetch(row + k * warps, k);
  for (int i = 0; row < rows; row += warps, ++i) {
    prefetch(row + (SLOTS - 1) * warps, (i + SLOTS - 1) % SLOTS);  // the slot row i - 1 used
    cp_async_wait<SLOTS - 1>();
    __syncwarp();
    const uint4* xv = buf + (i % SLOTS) * nvec;
    float v[PER][8];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int e = k * 32 + lane;
      if (e < nvec) {
        uint4 q = xv[e];
        uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = __half22float2(*reinterpret_cast<__half2*>(&w[j]));
          if (scaled) {
            f.x = __half2float(__float2half_rn(__fmul_rn(f.x, scale)));
            f.y = __half2float(__float2half_rn(__fmul_rn(f.y, scale)));
          }
          v[k][2 * j] = f.x;
          v[k][2 * j + 1] = f.y;
          m = row_max(row_max(m, f.x), f.y);
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = row_max(m, __shfl_xor_sync(0xffffffffu, m, o));
    const ShiftLog2 ml = shift_log2(m);
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int e = k * 32 + lane;
      if (e < nvec) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[k][j] = exp_shifted(v[k][j], ml);
          s = __fadd_rn(s, v[k][j]);
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    const float inv = __fdiv_rn(1.0f, s);
    uint4* yv = reinterpret_cast<uint4*>(y + row * reduce);
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int e = k * 32 + lane;
      if (e < nvec) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          __half2 h = __floats2half2_rn(__fmul_rn(v[k][2 * j], inv), __fmul_rn(v[k][2 * j + 1], inv));
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        yv[e] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    __syncwarp();  // this slot is refilled at the next row
  }
  cp_async_wait<0>();
}

// One block per row for long unit-stride rows: three passes through L2.
template <typename T, typename U>
__global__ void __launch_bounds__(512) softmax_block_rows(const T* x, U* y, RowSpace rs, int64_t rows,
                                                          int64_t reduce, int64_t rsx, int64_t rsy,
                                                          float scale, bool scaled) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    int64_t ox, oy;
    row_offsets(rs, row, ox, oy);
    float m = -INFINITY;
    for (int64_t e = threadIdx.x; e < reduce; e += blockDim.x)
      m = nan_max(m, load_scaled(x, ox + e * rsx, scale, scaled));
    for (int o = 16; o; o >>= 1) m = nan_max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
      for (int o = 16; o; o >>= 1) t = nan_max(t, __shfl_xor_sync(0xffffffffu, t, o));
      if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    m = red[0];
    __syncthreads();
    float s = 0.0f;
    for (int64_t e = threadIdx.x; e < reduce; e += blockDim.x)
      s = __fadd_rn(s, exp_fast(__fsub_rn(load_scaled(x, ox + e * rsx, scale, scaled), m)));
    for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
      for (int o = 16; o; o >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
      if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = __fdiv_rn(1.0f, red[0]);
    __syncthreads();
    for (int64_t e = threadIdx.x; e < reduce; e += blockDim.x)
      store_out(y, oy + e * rsy,
                __fmul_rn(exp_fast(__fsub_rn(load_scaled(x, ox + e * rsx, scale, scaled), m)), inv));
  }
}

// One thread per row for strided reductions (rows enumerated innermost-first,
// so neighbouring threads touch neighbouring addresses when a unit stride exists).
template <typename T, typename U>
__global__ void __launch_bounds__(256) softmax_thread_rows(const T* x, U* y, RowSpace rs, int64_t rows,
                                                           int64_t reduce, int64_t rsx, int64_t rsy,
                                                           float scale, bool scaled) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; row < rows; row += stride) {
    int64_t ox, oy;
    row_offsets(rs, row, ox, oy);
    float m = -INFINITY;
    for (int64_t e = 0; e < reduce; ++e) m = nan_max(m, load_scaled(x, ox + e * rsx, scale, scaled));
    float s = 0.0f;
    for (int64_t e = 0; e < reduce; ++e)
      s = __fadd_rn(s, exp_fast(__fsub_rn(load_scaled(x, ox + e * rsx, scale, scaled), m)));
    const float inv = __fdiv_rn(1.0f, s);
    for (int64_t e = 0; e < reduce; ++e)
      store_out(y, oy + e * rsy,
                __fmul_rn(exp_fast(__fsub_rn(load_scaled(x, ox + e * rsx, scale, scaled), m)), inv));
  }
}

// ------------------------------------------------------------ DFL decode

constexpr int kMaxLevels = 8;
struct Levels {
  int count;
  int64_t start[kMaxLevels];
  int64_t width[kMaxLevels];
  float stride[kMaxLevels];
};

__device__ __forceinline__ float h16(float v) { return __half2float(__float2half_rn(v)); }

// Round a probability p in [0, 1] (or NaN) to the nearest fp16 value, ties to
// even, without conversion instructions: on the fp32 bits for the fp16 normal
// range (drop 13 mantissa bits), by adding and removing 0.5 below it (fp32
// spacing at 0.5 is the fp16 subnormal quantum 2^-24).
__device__ __forceinline__ float round_prob_h16(float p) {
  if (p < 6.103515625e-05f) return __fsub_rn(__fadd_rn(p, 0.5f), 0.5f);
  uint32_t b = __float_as_uint(p);
  b = (b + 0x0fffu + ((b >> 13) & 1u)) & 0xffffe000u;
  return __uint_as_float(b);
}

// 16-bin softmax of one side (fp16 probabilities, as the separate softmax op
// stores them) followed by the arange(16) expectation rounded to fp16.
__device__ __forceinline__ float dfl_side(const float (&v)[16]) {
  float m = v[0];
#pragma unroll
  for (int i = 1; i < 16; ++i) m = row_max(m, v[i]);  // NaN/inf reach the sum below
  const ShiftLog2 ml = shift_log2(m);
  float e[16], s = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    e[i] = exp_shifted(v[i], ml);
    s = __fadd_rn(s, e[i]);
  }
  const float inv = __fdiv_rn(1.0f, s);
  float d = 0.0f;
#pragma unroll
  for (int i = 1; i < 16; ++i) d = __fmaf_rn(round_prob_h16(__fmul_rn(e[i], inv)), (float)i, d);
  return h16(d);
}

template <int APT>
__global__ void __launch_bounds__(128) dfl_decode(const __half* box, int64_t box_bs, int64_t box_cs,
                                                  const __half* cls, int64_t cls_bs, int64_t cls_cs,
                                                  int64_t n, int64_t nc, int64_t anchors, Levels lv,
                                                  bool xywh, __half* out, __half* dist_out) {
  const int64_t groups = (anchors + APT - 1) / APT;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n * groups; t += stride) {
    const int64_t b = t / groups;
    const int64_t a0 = (t % groups) * APT;
    const __half* bx = box + b * box_bs + a0;
    __half* o = out + b * (4 + nc) * anchors + a0;
    float dist[4][APT];
#pragma unroll
    for (int sd = 0; sd < 4; ++sd) {
      float v[APT][16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const __half* p = bx + (sd * 16 + i) * box_cs;
        if constexpr (APT == 2) {
          float2 f = __half22float2(*reinterpret_cast<const __half2*>(p));
          v[0][i] = f.x;
          v[1][i] = f.y;
        } else {
          v[0][i] = __half2float(*p);
        }
      }
#pragma unroll
      for (int k = 0; k < APT; ++k) dist[sd][k] = dfl_side(v[k]);
    }
    float res[4][APT];
#pragma unroll
    for (int k = 0; k < APT; ++k) {
      int64_t a = a0 + k;
      if (a >= anchors) {
        res[0][k] = res[1][k] = res[2][k] = res[3][k] = 0.0f;
        continue;
      }
      if (dist_out) {
#pragma unroll
        for (int sd = 0; sd < 4; ++sd) dist_out[(b * 4 + sd) * anchors + a] = __float2half_rn(dist[sd][k]);
      }
      int l = 0;
      while (l + 1 < lv.count && a >= lv.start[l + 1]) ++l;
      int64_t local = a - lv.start[l];
      float ax = h16((float)(local % lv.width[l]) + 0.5f);
      float ay = h16((float)(local / lv.width[l]) + 0.5f);
      float st = lv.stride[l];
      float lx = h16(__fsub_rn(ax, dist[0][k])), ly = h16(__fsub_rn(ay, dist[1][k]));
      float ux = h16(__fadd_rn(ax, dist[2][k])), uy = h16(__fadd_rn(ay, dist[3][k]));
      float q[4];
      if (xywh) {
        q[0] = h16(__fdiv_rn(h16(__fadd_rn(lx, ux)), 2.0f));
        q[1] = h16(__fdiv_rn(h16(__fadd_rn(ly, uy)), 2.0f));
        q[2] = h16(__fsub_rn(ux, lx));
        q[3] = h16(__fsub_rn(uy, ly));
      } else {
        q[0] = lx; q[1] = ly; q[2] = ux; q[3] = uy;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) res[c][k] = __fmul_rn(q[c], st);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if constexpr (APT == 2) {
        *reinterpret_cast<__half2*>(o + c * anchors) = __floats2half2_rn(res[c][0], res[c][1]);
      } else {
        o[c * anchors] = __float2half_rn(res[c][0]);
      }
    }
    const __half* cx = cls + b * cls_bs + a0;
    for (int64_t c = 0; c < nc; ++c) {
      if constexpr (APT == 2) {
        uint32_t w = *reinterpret_cast<const uint32_t*>(cx + c * cls_cs);
        uint32_t r = unary_h2_fast<false>(w);
        *reinterpret_cast<uint32_t*>(o + (4 + c) * anchors) = r;
      } else {
        reinterpret_cast<uint16_t*>(o)[(4 + c) * anchors] =
            sigmoid_h_fast(reinterpret_cast<const uint16_t*>(cx)[c * cls_cs]);
      }
    }
  }
}

// dfl_side for two anchors at once: w[i] holds bin i of both anchors as a half2.
// Same rounding points: fp16 probabilities (one packed conversion per bin pair),
// fp32 expectation accumulated over bins 1..15 in order, rounded to fp16.  The
// two anchors' fp32 chains run as the halves of paired f32x2 operations.
__device__ __forceinline__ float2 dfl_side2(const uint32_t (&w)[16]) {
  float2 v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
  float m0 = v[0].x, m1 = v[0].y;
#pragma unroll
  for (int i = 1; i < 16; ++i) {
    m0 = row_max(m0, v[i].x);
    m1 = row_max(m1, v[i].y);
  }
  const ShiftLog2 l0 = shift_log2(m0), l1 = shift_log2(m1);
  const unsigned long long log2e = f2_pack(1.44269504088896341f, 1.44269504088896341f);
  const unsigned long long shift = f2_pack(-l0.hi, -l1.hi);
  unsigned long long e[16], sum = f2_pack(0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {  // exp(v - m') per anchor, as exp_shifted does
    const float2 arg = f2_unpack(f2_fma(f2_pack(v[i].x, v[i].y), log2e, shift));
    e[i] = f2_pack(ex2_approx(arg.x), ex2_approx(arg.y));
    sum = f2_add(sum, e[i]);
  }
  const float2 s = f2_unpack(sum);
  const unsigned long long inv = f2_pack(__fdiv_rn(1.0f, s.x), __fdiv_rn(1.0f, s.y));
  unsigned long long d = f2_pack(0.0f, 0.0f);
#pragma unroll
  for (int i = 1; i < 16; ++i) {
    const float2 pr = f2_unpack(f2_mul(e[i], inv));
    const float2 p = __half22float2(__floats2half2_rn(pr.x, pr.y));
    d = f2_fma(f2_pack(p.x, p.y), f2_pack((float)i, (float)i), d);
  }
  const float2 dd = f2_unpack(d);
  return make_float2(h16(dd.x), h16(dd.y));
}

// Box half of the decode for 8-aligned anchors: a block walks 128-anchor tiles
// of the 64 box rows; the next tile streams into the other shared-memory buffer
// with cp.async while this one is reduced.  Thread (side, anchor pair) runs the
// two DFL reductions from half2 reads; thread (anchor) then decodes its four
// coordinates; the 4 x 128 output tile leaves with 16-byte stores.  Index math
// is 32-bit (anchors < 2^30).  The class rows are a separate elementwise sigmoid
// (unary_rows2_f16).
constexpr int kTileA = 128;

__global__ void __launch_bounds__(256) dfl_box_tiled(const __half* box, int64_t box_bs, int64_t box_cs,
                                                     int n, int anchors, Levels lv, bool xywh,
                                                     __half* out, int64_t out_bs, __half* dist_out) {
  __shared__ __align__(16) uint16_t in_box[2][64][kTileA];
  __shared__ float dist[4][kTileA];
  __shared__ __align__(16) uint16_t out_box[4][kTileA];
  const int tiles = (anchors + kTileA - 1) / kTileA;
  const int jobs = n * tiles;
  const int tid = threadIdx.x;
  auto issue = [&](int job, int buf) {
    if (job < jobs) {
      const int b = job / tiles, a0 = (job - b * tiles) * kTileA;
      const int vecs = (anchors - a0 < kTileA ? anchors - a0 : kTileA) / 8;
      const __half* src = box + (int64_t)b * box_bs + a0;
#pragma unroll
      for (int v = tid; v < 64 * (kTileA / 8); v += 256) {
        const int row = v / (kTileA / 8), c = v % (kTileA / 8);
        if (c < vecs) cp_async16(&in_box[buf][row][c * 8], src + row * box_cs + c * 8);
      }
    }
    cp_async_commit();
  };
  int buf = 0;
  issue(blockIdx.x, 0);
  for (int job = blockIdx.x; job < jobs; job += gridDim.x, buf ^= 1) {
    issue(job + gridDim.x, buf ^ 1);  // that buffer's last reader finished before the previous sync
    cp_async_wait<1>();
    __syncthreads();
    const int b = job / tiles, a0 = (job - b * tiles) * kTileA;
    const int vecs = (anchors - a0 < kTileA ? anchors - a0 : kTileA) / 8;
    {  // DFL: thread -> (side, anchor pair)
      const int side = tid >> 6, a = (tid & 63) * 2;
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = *reinterpret_cast<const uint32_t*>(&in_box[buf][side * 16 + i][a]);
      const float2 d = dfl_side2(w);
      dist[side][a] = d.x;
      dist[side][a + 1] = d.y;
    }
    __syncthreads();
    if (tid < kTileA) {  // box decode: thread -> anchor
      const int a = tid, idx = a0 + a;
      if (dist_out && idx < anchors) {  // trace: the four DFL distances of this anchor
#pragma unroll
        for (int side = 0; side < 4; ++side)
          dist_out[((int64_t)b * 4 + side) * anchors + idx] = __float2half_rn(dist[side][a]);
      }
      int lstart = 0, lwidth = (int)lv.width[0];
      float lstride = lv.stride[0];
#pragma unroll
      for (int k = 1; k < kMaxLevels; ++k) {  // starts increase: the last level begun holds idx
        if (k < lv.count && idx >= (int)lv.start[k]) {
          lstart = (int)lv.start[k];
          lwidth = (int)lv.width[k];
          lstride = lv.stride[k];
        }
      }
      const int local = idx - lstart;
      const int gy = local / lwidth;
      const float ax = h16((float)(local - gy * lwidth) + 0.5f);
      const float ay = h16((float)gy + 0.5f);
      const float lx = h16(__fsub_rn(ax, dist[0][a])), ly = h16(__fsub_rn(ay, dist[1][a]));
      const float ux = h16(__fadd_rn(ax, dist[2][a])), uy = h16(__fadd_rn(ay, dist[3][a]));
      float q[4];
      if (xywh) {  // x / 2 == x * 0.5 exactly (both are the correctly rounded half)
        q[0] = h16(__fmul_rn(h16(__fadd_rn(lx, ux)), 0.5f));
        q[1] = h16(__fmul_rn(h16(__fadd_rn(ly, uy)), 0.5f));
        q[2] = h16(__fsub_rn(ux, lx));
        q[3] = h16(__fsub_rn(uy, ly));
      } else {
        q[0] = lx;
        q[1] = ly;
        q[2] = ux;
        q[3] = uy;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) out_box[c][a] = hbits(__float2half_rn(__fmul_rn(q[c], lstride)));
    }
    __syncthreads();
    if (tid < 4 * (kTileA / 8)) {
      const int row = tid / (kTileA / 8), c = tid % (kTileA / 8);
      if (c < vecs)
        *reinterpret_cast<uint4*>(out + (int64_t)b * out_bs + (int64_t)row * anchors + a0 + c * 8) =
            *reinterpret_cast<const uint4*>(&out_box[row][c * 8]);
    }
  }
  cp_async_wait<0>();
}

template <typename T, typename U>
ttn_status launch_softmax(const ttn_tensor* x, const ttn_tensor* y, int dim, float scale,
                          cudaStream_t s) {
  const bool scaled = scale != 1.0f;
  RowSpace rs;
  rs.ndim = 0;
  int64_t rows = 1;
  // non-reduced dims, innermost first, merging where both views allow
  for (int d = x->ndim - 1; d >= 0; --d) {
    if (d == dim || x->sizes[d] == 1) continue;
    rows *= x->sizes[d];
    if (rs.ndim && rs.sx[rs.ndim - 1] * rs.size[rs.ndim - 1] == x->strides[d] &&
        rs.sy[rs.ndim - 1] * rs.size[rs.ndim - 1] == y->strides[d]) {
      rs.size[rs.ndim - 1] *= x->sizes[d];
    } else {
      if (rs.ndim == 7) return fail(TTN_UNSUPPORTED, "ttn_softmax: too many dims");
      rs.size[rs.ndim] = x->sizes[d];
      rs.sx[rs.ndim] = x->strides[d];
      rs.sy[rs.ndim] = y->strides[d];
      ++rs.ndim;
    }
  }
  for (int d = 0; d < x->ndim; ++d)
    if (x->sizes[d] == 0) return TTN_OK;
  const int64_t reduce = x->ndim ? x->sizes[dim] : 1;
  const int64_t rsx = x->ndim ? x->strides[dim] : 1, rsy = y->ndim ? y->strides[dim] : 1;
  if (reduce == 0 || rows == 0) return TTN_OK;
  const T* xp = (const T*)x->data;
  U* yp = (U*)y->data;
  if (rsx == 1 && rsy == 1 && reduce <= 1024) {
    if constexpr (sizeof(T) == 2 && sizeof(U) == 2) {
      bool vec = reduce % 8 == 0 && ((uintptr_t)xp & 15u) == 0 && ((uintptr_t)yp & 15u) == 0;
      for (int d = 0; d < rs.ndim && vec; ++d) vec = rs.sx[d] % 8 == 0 && rs.sy[d] % 8 == 0;
      bool packed = vec && rs.ndim <= 1 && (rs.ndim == 0 || (rs.sx[0] == reduce && rs.sy[0] == reduce));
      if (packed && rows >= 1024) {  // contiguous rows: cp.async double buffering
        int nvec = (int)(reduce / 8);
        int per = nvec <= 32 ? 1 : nvec <= 64 ? 2 : 4;
        const int slots = per <= 2 ? 4 : 2;
        size_t smem = (size_t)kRowsWarps * slots * nvec * 16;
        const void* fn = per == 1 ? (const void*)softmax_rows_pipelined<1, 4>
                       : per == 2 ? (const void*)softmax_rows_pipelined<2, 4>
                                  : (const void*)softmax_rows_pipelined<4, 2>;
        TTN_TRY(ensure_dynamic_smem(fn, (int)smem));
        unsigned grid = (unsigned)(sm_count() * resident_blocks(fn, kRowsWarps * 32, smem));
        int64_t need = (rows + kRowsWarps - 1) / kRowsWarps;
        if ((int64_t)grid > need) grid = (unsigned)need;
        if (per == 1)
          softmax_rows_pipelined<1, 4><<<grid, kRowsWarps * 32, smem, s>>>((const uint16_t*)xp, (uint16_t*)yp,
                                                                       rows, (int)reduce, scale, scaled);
        else if (per == 2)
          softmax_rows_pipelined<2, 4><<<grid, kRowsWarps * 32, smem, s>>>((const uint16_t*)xp, (uint16_t*)yp,
                                                                       rows, (int)reduce, scale, scaled);
        else
          softmax_rows_pipelined<4, 2><<<grid, kRowsWarps * 32, smem, s>>>((const uint16_t*)xp, (uint16_t*)yp,
                                                                       rows, (int)reduce, scale, scaled);
        return launch_check("ttn_softmax");
      }
      if (vec) {
        unsigned grid = grid_for(rows, 8, 16);
        int nvec = (int)(reduce / 8);
        if (nvec <= 32)
          softmax_warp_rows_h8<1><<<grid, 256, 0, s>>>((const uint16_t*)xp, (uint16_t*)yp, rs, rows,
                                                       (int)reduce, scale, scaled);
        else if (nvec <= 64)
          softmax_warp_rows_h8<2><<<grid, 256, 0, s>>>((const uint16_t*)xp, (uint16_t*)yp, rs, rows,
                                                       (int)reduce, scale, scaled);
        else
          softmax_warp_rows_h8<4><<<grid, 256, 0, s>>>((const uint16_t*)xp, (uint16_t*)yp, rs, rows,
                                                       (int)reduce, scale, scaled);
        return launch_check("ttn_softmax");
      }
    }
    unsigned grid = grid_for(rows, 8, 16);
    if (reduce <= 128)
      softmax_warp_rows<T, U, 4><<<grid, 256, 0, s>>>(xp, yp, rs, rows, (int)reduce, scale, scaled);
    else if (reduce <= 256)
      softmax_warp_rows<T, U, 8><<<grid, 256, 0, s>>>(xp, yp, rs, rows, (int)reduce, scale, scaled);
    else if (reduce <= 512)
      softmax_warp_rows<T, U, 16><<<grid, 256, 0, s>>>(xp, yp, rs, rows, (int)reduce, scale, scaled);
    else
      softmax_warp_rows<T, U, 32><<<grid, 256, 0, s>>>(xp, yp, rs, rows, (int)reduce, scale, scaled);
    return launch_check("ttn_softmax");
  }
  if (rsx == 1 && rsy == 1) {
    unsigned grid = grid_for(rows, 1, 4);
    softmax_block_rows<T, U><<<grid, 512, 0, s>>>(xp, yp, rs, rows, reduce, rsx, rsy, scale, scaled);
    return launch_check("ttn_softmax");
  }
  unsigned grid = grid_for(rows, 256);
  softmax_thread_rows<T, U><<<grid, 256, 0, s>>>(xp, yp, rs, rows, reduce, rsx, rsy, scale, scaled);
  return launch_check("ttn_softmax");
}

}  // namespace
}  // namespace ttn

using namespace ttn;

extern "C" {

ttn_status ttn_softmax(const ttn_tensor* x, int32_t dim, float scale, const ttn_tensor* y,
                       ttn_stream stream) {
  const char* name = "ttn_softmax";
  TTN_TRY(validate(x, name));
  TTN_TRY(validate(y, name));
  if (!same_sizes(x, y)) return fail(TTN_INVALID_ARG, "%s: x and y sizes differ", name);
  if (x->ndim == 0 ? (dim != 0 && dim != -1) : (dim < 0 || dim >= x->ndim))
    return fail(TTN_INVALID_ARG, "%s: dim %d out of range", name, dim);
  if (x->ndim == 0) dim = 0;
  if (x->dtype == TTN_F32 && y->dtype == TTN_F16)
    return fail(TTN_INVALID_ARG, "%s: float32 input cannot produce float16 output", name);
  if (!(scale == scale)) return fail(TTN_INVALID_ARG, "%s: scale is NaN", name);
  cudaStream_t s = (cudaStream_t)stream;
  if (x->dtype == TTN_F16 && y->dtype == TTN_F16) return launch_softmax<uint16_t, uint16_t>(x, y, dim, scale, s);
  if (x->dtype == TTN_F16) return launch_softmax<uint16_t, float>(x, y, dim, scale, s);
  return launch_softmax<float, float>(x, y, dim, scale, s);
}

ttn_status ttn_dfl_decode_trace_f16(const void* box, int64_t box_bs, int64_t box_cs, const void* cls,
                                    int64_t cls_bs, int64_t cls_cs, int64_t n, int64_t nc,
                                    int32_t levels, const int64_t* heights, const int64_t* widths,
                                    const float* strides, int32_t xywh, void* out, void* distances,
                                    ttn_stream stream) {
  const char* name = distances ? "ttn_dfl_decode_trace_f16" : "ttn_dfl_decode_f16";
  if (n < 0 || nc < 0) return fail(TTN_INVALID_ARG, "%s: negative size", name);
  if (levels < 1 || levels > kMaxLevels || !heights || !widths || !strides)
    return fail(TTN_INVALID_ARG, "%s: 1..%d levels with heights/widths/strides", name, kMaxLevels);
  Levels lv;
  lv.count = levels;
  int64_t anchors = 0;
  for (int l = 0; l < levels; ++l) {
    if (heights[l] <= 0 || widths[l] <= 0 || !(strides[l] > 0.0f))
      return fail(TTN_INVALID_ARG, "%s: level %d has a non-positive size or stride", name, l);
    if (heights[l] > 1024 || widths[l] > 1024)
      return fail(TTN_UNSUPPORTED, "%s: grid side > 1024 is not exact in fp16 anchors", name);
    lv.start[l] = anchors;
    lv.width[l] = widths[l];
    lv.stride[l] = strides[l];
    anchors += heights[l] * widths[l];
  }
  if (!n || !anchors) return TTN_OK;
  if (!box || !out || (nc && !cls)) return fail(TTN_INVALID_ARG, "%s: null pointer", name);
  bool pair = anchors % 2 == 0 && ((uintptr_t)box & 3u) == 0 && ((uintptr_t)out & 3u) == 0 &&
              box_bs % 2 == 0 && box_cs % 2 == 0 &&
              (!nc || (((uintptr_t)cls & 3u) == 0 && cls_bs % 2 == 0 && cls_cs % 2 == 0));
  cudaStream_t s = (cudaStream_t)stream;
  bool tiled = anchors % 8 == 0 && anchors < ((int64_t)1 << 30) &&
               n * ((anchors + kTileA - 1) / kTileA) < ((int64_t)1 << 31) && ((uintptr_t)box & 15u) == 0 &&
               ((uintptr_t)out & 15u) == 0 && box_bs % 8 == 0 && box_cs % 8 == 0 &&
               (!nc || (((uintptr_t)cls & 15u) == 0 && cls_bs % 8 == 0 && cls_cs % 8 == 0));
  if (tiled) {
    int64_t jobs = n * ((anchors + kTileA - 1) / kTileA);
    unsigned grid = resident_grid(dfl_box_tiled, 256, 0, jobs, 1);
    // the class sigmoid (HBM-bound) runs on a forked branch beside the box
    // reduction (issue-bound); both read disjoint rows and write disjoint rows
    cudaStream_t aux = s;
    if (nc) TTN_TRY(branch_fork(s, &aux));
    ttn_status st = nc ? unary_rows2_f16(1, (const uint16_t*)cls, cls_bs, cls_cs,
                                         (uint16_t*)out + 4 * anchors, (4 + nc) * anchors, anchors, n,
                                         nc, anchors, aux)
                       : TTN_OK;
    dfl_box_tiled<<<grid, 256, 0, s>>>((const __half*)box, box_bs, box_cs, (int)n, (int)anchors, lv,
                                       xywh != 0, (__half*)out, (4 + nc) * anchors, (__half*)distances);
    ttn_status launched = launch_check(name);
    ttn_status joined = nc ? branch_join(s) : TTN_OK;
    return st != TTN_OK ? st : launched != TTN_OK ? launched : joined;
  }
  if (pair) {
    int64_t work = n * (anchors / 2);
    dfl_decode<2><<<grid_for(work, 128, 16), 128, 0, s>>>(
        (const __half*)box, box_bs, box_cs, (const __half*)cls, cls_bs, cls_cs, n, nc, anchors, lv,
        xywh != 0, (__half*)out, (__half*)distances);
  } else {
    int64_t work = n * anchors;
    dfl_decode<1><<<grid_for(work, 128, 16), 128, 0, s>>>(
        (const __half*)box, box_bs, box_cs, (const __half*)cls, cls_bs, cls_cs, n, nc, anchors, lv,
        xywh != 0, (__half*)out, (__half*)distances);
  }
  return launch_check(name);
}

ttn_status ttn_dfl_decode_f16(const void* box, int64_t box_bs, int64_t box_cs, const void* cls,
                              int64_t cls_bs, int64_t cls_cs, int64_t n, int64_t nc,
                              int32_t levels, const int64_t* heights, const int64_t* widths,
                              const float* strides, int32_t xywh, void* out, ttn_stream stream) {
  return ttn_dfl_decode_trace_f16(box, box_bs, box_cs, cls, cls_bs, cls_cs, n, nc, levels, heights, widths,
                                  strides, xywh, out, nullptr, stream);
}

}  // extern "C"
