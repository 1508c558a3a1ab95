// Spatial/layout ops over fp16 feature maps: NC1HWC0 <-> NCHW transposes,
// nearest-2x upsample, odd-kernel stride-1 max-pool and the fused SPPF tail.
//
// Layout conversions stage a 64-pixel x 16-channel tile in shared memory so
// both the 32-byte pixel vectors of NC1HWC0 and the 128-byte channel rows of
// NCHW move as 16-byte accesses.  Max-pool stages a band of rows (plus the
// halo) in shared memory and runs the separable window horizontally, then
// vertically, which reproduces CPU F.max_pool2d's row-major scan exactly: the
// first maximum wins among equal values (so -0 vs +0 keeps the earlier one)
// and the last NaN in scan order wins, quieted as CPU's fp32 round trip does.
#include "common.cuh"

namespace ttn {
namespace {

constexpr int kPix = 64;  // pixels per layout tile

// x: [n, c1, hw, 16] -> y[b*ybs + c*ycs + p] for c < channels.
__global__ void __launch_bounds__(128) blocked_to_nchw(const uint16_t* x, int64_t n, int64_t c1,
                                                       int64_t hw, int64_t channels, uint16_t* y,
                                                       int64_t ybs, int64_t ycs, bool vector_out) {
  __shared__ __align__(16) uint16_t tile[16][kPix + 8];
  const int64_t tiles = (hw + kPix - 1) / kPix;
  for (int64_t job = blockIdx.x; job < n * c1 * tiles; job += gridDim.x) {
    int64_t plane = job / tiles;  // b*c1 + cb
    int64_t p0 = (job % tiles) * kPix;
    int64_t b = plane / c1, cb = plane % c1;
    int count = (int)(hw - p0 < kPix ? hw - p0 : kPix);
    const uint16_t* src = x + (plane * hw + p0) * 16;
    // load: thread t reads pixel t/2, channels (t&1)*8 .. +8
    for (int v = threadIdx.x; v < count * 2; v += blockDim.x) {
      uint4 q = reinterpret_cast<const uint4*>(src)[v];
      int p = v >> 1, c = (v & 1) * 8;
      uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        tile[c + 2 * k][p] = (uint16_t)(w[k] & 0xffffu);
        tile[c + 2 * k + 1][p] = (uint16_t)(w[k] >> 16);
      }
    }
    __syncthreads();
    int valid = (int)(channels - cb * 16 < 16 ? channels - cb * 16 : 16);
    if (vector_out && count == kPix) {
      // 16 channels x 8 vectors of 8 pixels
      int c = threadIdx.x >> 3, v = threadIdx.x & 7;
      if (c < valid) {
        uint16_t* dst = y + b * ybs + (cb * 16 + c) * ycs + p0 + v * 8;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(&tile[c][v * 8]);
      }
    } else {
      for (int e = threadIdx.x; e < valid * count; e += blockDim.x) {
        int c = e / count, p = e % count;
        y[b * ybs + (cb * 16 + c) * ycs + p0 + p] = tile[c][p];
      }
    }
    __syncthreads();
  }
}

// Register-transpose variant for hw % 4 == 0 and 8-byte aligned channel rows:
// one thread per (plane, 4-pixel group) takes 4 pixels x 16 lanes (128 B) and
// writes 16 channel rows of 4 pixels (8 B each; consecutive threads fill
// consecutive 8 B of a row).  The warp loads its 32 groups together through a
// shared-memory tile (one 512-byte coalesced load per instruction instead of 32
// separate 128-byte runs); the 4x16 fp16 transpose is 32 byte permutes.
__global__ void __launch_bounds__(256) blocked_to_nchw_regs(const uint4* x, int64_t n, int64_t c1,
                                                            int64_t hw, int64_t channels, uint16_t* y,
                                                            int64_t ybs, int64_t ycs) {
  // A warp's 32 (plane, 4-pixel) items are one contiguous 4 KB of x (planes are
  // adjacent), loaded with consecutive lanes on consecutive 16-byte vectors into a
  // per-warp tile; vector j sits at j ^ ((j >> 3) & 7), so both the loads' stores
  // (8 lanes on 8 consecutive vectors) and each lane's read-back of its own 8
  // vectors (8 lanes 8 vectors apart) cover all 8 bank groups.
  __shared__ uint4 tile[8][256];
  uint4* mine = tile[threadIdx.x >> 5];
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  const int64_t groups = hw / 4;
  const int64_t total = n * c1 * groups;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31); t0 < total; t0 += stride) {
    const int64_t vecs = (total - t0) * 8 < 256 ? (total - t0) * 8 : 256;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = k * 32 + lane;
      if (j < vecs) mine[j ^ ((j >> 3) & 7)] = x[t0 * 8 + j];
    }
    __syncwarp();
    const int64_t t = t0 + lane;
    if (t < total) {
      const int64_t plane = t / groups, g = t - plane * groups;
      const int64_t b = plane / c1, cb = plane - b * c1;
      uint32_t in[4][8];  // [pixel][channel pair]
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint4 lo = mine[(8 * lane + 2 * p) ^ (lane & 7)], hi = mine[(8 * lane + 2 * p + 1) ^ (lane & 7)];
        in[p][0] = lo.x;
        in[p][1] = lo.y;
        in[p][2] = lo.z;
        in[p][3] = lo.w;
        in[p][4] = hi.x;
        in[p][5] = hi.y;
        in[p][6] = hi.z;
        in[p][7] = hi.w;
      }
      const int valid = (int)(channels - cb * 16 < 16 ? channels - cb * 16 : 16);
      uint16_t* dst = y + b * ybs + (cb * 16) * ycs + g * 4;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        if (c < valid) {
          const uint32_t sel = (c & 1) ? 0x7632u : 0x5410u;  // high or low lane of each word
          uint2 o;
          o.x = __byte_perm(in[0][c >> 1], in[1][c >> 1], sel);
          o.y = __byte_perm(in[2][c >> 1], in[3][c >> 1], sel);
          *reinterpret_cast<uint2*>(dst + c * ycs) = o;
        }
      }
    }
    __syncwarp();  // the tile is refilled next round
  }
}

// x: NCHW [n, channels, hw] -> y: [n, ceil(channels/16), hw, 16], zero-padded.
__global__ void __launch_bounds__(128) nchw_to_blocked(const uint16_t* x, int64_t n,
                                                       int64_t channels, int64_t hw, uint16_t* y,
                                                       bool vector_in) {
  __shared__ __align__(16) uint16_t tile[16][kPix + 8];
  const int64_t c1 = (channels + 15) / 16;
  const int64_t tiles = (hw + kPix - 1) / kPix;
  for (int64_t job = blockIdx.x; job < n * c1 * tiles; job += gridDim.x) {
    int64_t plane = job / tiles;
    int64_t p0 = (job % tiles) * kPix;
    int64_t b = plane / c1, cb = plane % c1;
    int count = (int)(hw - p0 < kPix ? hw - p0 : kPix);
    int valid = (int)(channels - cb * 16 < 16 ? channels - cb * 16 : 16);
    if (vector_in && count == kPix) {
      int c = threadIdx.x >> 3, v = threadIdx.x & 7;
      uint4 q = make_uint4(0, 0, 0, 0);
      if (c < valid)
        q = *reinterpret_cast<const uint4*>(x + (b * channels + cb * 16 + c) * hw + p0 + v * 8);
      *reinterpret_cast<uint4*>(&tile[c][v * 8]) = q;
    } else {
      for (int e = threadIdx.x; e < 16 * count; e += blockDim.x) {
        int c = e / count, p = e % count;
        tile[c][p] = c < valid ? x[(b * channels + cb * 16 + c) * hw + p0 + p] : (uint16_t)0;
      }
    }
    __syncthreads();
    uint16_t* dst = y + (plane * hw + p0) * 16;
    for (int v = threadIdx.x; v < count * 2; v += blockDim.x) {
      int p = v >> 1, c = (v & 1) * 8;
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        w[k] = (uint32_t)tile[c + 2 * k][p] | ((uint32_t)tile[c + 2 * k + 1][p] << 16);
      reinterpret_cast<uint4*>(dst)[v] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------- upsample

// NC1HWC0: each input 16-byte vector (half a pixel's 16 lanes) is written to the
// 4 output pixels it covers.  Images may sit at any 16-byte-multiple batch
// stride (x_bs, y_bs in uint4 units), e.g. inside a concat buffer.
__global__ void __launch_bounds__(256) upsample_blocked(const uint4* x, uint4* y, int64_t n,
                                                        int64_t c1, int64_t h, int64_t w,
                                                        int64_t x_bs, int64_t y_bs) {
  const int64_t per_image = c1 * h * w * 2;
  const int64_t nvec = n * per_image;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    int64_t b = v / per_image, local = v - b * per_image;
    uint4 q = x[b * x_bs + local];
    int64_t p = local >> 1;
    int j = (int)(local & 1);
    int64_t col = p % w, rest = p / w;
    int64_t row = rest % h, plane = rest / h;
    int64_t base = b * y_bs + ((plane * 2 * h + 2 * row) * 2 * w + 2 * col) * 2 + j;
    y[base] = q;
    y[base + 2] = q;
    y[base + 4 * w] = q;
    y[base + 4 * w + 2] = q;
  }
}

// upsample_blocked for launches below 2^31 vectors: the vector's (image, plane,
// row, column, half) from 32-bit multiply-high divisions instead of 64-bit ones.
__global__ void __launch_bounds__(256) upsample_blocked32(const uint4* x, uint4* y, uint32_t nvec,
                                                          FastDiv per_image, FastDiv hdiv, FastDiv wdiv,
                                                          int64_t x_bs, int64_t y_bs) {
  const uint32_t stride = gridDim.x * blockDim.x;
  const int64_t w = wdiv.d, h = hdiv.d;
  pdl_trigger();
  pdl_wait();
  for (uint32_t v = blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    const uint32_t b = per_image.div(v), local = v - b * per_image.d;
    const uint4 q = x[b * x_bs + local];
    const uint32_t p = local >> 1, j = local & 1;
    const uint32_t rest = wdiv.div(p), col = p - rest * wdiv.d;
    const uint32_t plane = hdiv.div(rest), row = rest - plane * hdiv.d;
    const int64_t base = b * y_bs + (((int64_t)plane * 2 * h + 2 * row) * 2 * w + 2 * col) * 2 + j;
    y[base] = q;
    y[base + 2] = q;
    y[base + 4 * w] = q;
    y[base + 4 * w + 2] = q;
  }
}

// NCHW with w % 4 == 0: read 4 input columns (8 bytes), write 8 output columns
// (16 bytes) to both output rows.
__global__ void __launch_bounds__(256) upsample_nchw_vec(const uint2* x, uint4* y, int64_t planes,
                                                         int64_t h, int64_t w4) {
  const int64_t nvec = planes * h * w4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    uint2 q = x[v];
    int64_t col = v % w4, rest = v / w4;
    uint32_t a = q.x & 0xffffu, b = q.x >> 16, c = q.y & 0xffffu, d = q.y >> 16;
    uint4 o = make_uint4(a | (a << 16), b | (b << 16), c | (c << 16), d | (d << 16));
    int64_t row0 = rest * 2;  // output row of input row `rest` (= plane*h + row)
    y[row0 * w4 + col] = o;
    y[(row0 + 1) * w4 + col] = o;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) upsample_nchw_scalar(const T* x, T* y, int64_t planes,
                                                            int64_t h, int64_t w) {
  const int64_t total = planes * h * w * 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += stride) {
    int64_t col = o % (2 * w), rest = o / (2 * w);
    int64_t row = rest % (2 * h), plane = rest / (2 * h);
    y[o] = x[(plane * h + row / 2) * w + col / 2];
  }
}

// --------------------------------------------------------------- maxpool

// CPU F.max_pool2d update rule on raw bits: take v when v > m or v is NaN.
template <typename T>
struct PoolBits;
template <>
struct PoolBits<uint16_t> {
  static __device__ __forceinline__ float value(uint16_t b) { return __half2float(hfrom(b)); }
  static __device__ __forceinline__ uint16_t neg_inf() { return 0xfc00u; }
  static __device__ __forceinline__ uint16_t finish(uint16_t b) { return hnan_bits(b) ? hquiet(b) : b; }
};
template <>
struct PoolBits<uint32_t> {
  static __device__ __forceinline__ float value(uint32_t b) { return __uint_as_float(b); }
  static __device__ __forceinline__ uint32_t neg_inf() { return 0xff800000u; }
  static __device__ __forceinline__ uint32_t finish(uint32_t b) {
    return ((b & 0x7fffffffu) > 0x7f800000u) ? (b | 0x00400000u) : b;
  }
};

template <typename T>
__device__ __forceinline__ void pool_update(T& m, float& mv, T v) {
  float vv = PoolBits<T>::value(v);
  if (vv > mv || vv != vv) {
    m = v;
    mv = vv;
  }
}

// One block = one plane band: output rows [r0, r0+rows) of plane `plane`,
// `lanes` interleaved channels per pixel (16 for NC1HWC0, 1 for NCHW).
// smem: in[(rows+2r) x w x lanes], hmax[(rows+2r) x w x lanes].
template <typename T>
__global__ void __launch_bounds__(256) maxpool_band(const T* x, T* y, int64_t planes, int h, int w,
                                                    int lanes, int radius, int band) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* in = reinterpret_cast<T*>(smem_raw);
  const int rows_max = band + 2 * radius;
  T* hmax = in + (size_t)rows_max * w * lanes;
  const int bands = (h + band - 1) / band;
  const int row_elems = w * lanes;
  for (int64_t job = blockIdx.x; job < planes * bands; job += gridDim.x) {
    int64_t plane = job / bands;
    int r0 = (int)(job % bands) * band;
    int rows = h - r0 < band ? h - r0 : band;
    int in0 = r0 - radius > 0 ? r0 - radius : 0;
    int in1 = r0 + rows + radius < h ? r0 + rows + radius : h;
    int in_rows = in1 - in0;
    const T* src = x + (plane * h + in0) * (int64_t)row_elems;
    for (int e = threadIdx.x; e < in_rows * row_elems; e += blockDim.x) in[e] = src[e];
    __syncthreads();
    // horizontal pass over every staged row
    for (int e = threadIdx.x; e < in_rows * row_elems; e += blockDim.x) {
      int lane = e % lanes, col = (e / lanes) % w, row = e / row_elems;
      int c0 = col - radius > 0 ? col - radius : 0;
      int c1 = col + radius < w - 1 ? col + radius : w - 1;
      T m = PoolBits<T>::neg_inf();
      float mv = -INFINITY;
      const T* r = in + row * row_elems + lane;
      for (int c = c0; c <= c1; ++c) pool_update(m, mv, r[c * lanes]);
      hmax[e] = m;
    }
    __syncthreads();
    // vertical pass for the band's output rows
    T* dst = y + (plane * h + r0) * (int64_t)row_elems;
    for (int e = threadIdx.x; e < rows * row_elems; e += blockDim.x) {
      int row = r0 + e / row_elems, rest = e % row_elems;
      int q0 = row - radius > 0 ? row - radius : 0;
      int q1 = row + radius < h - 1 ? row + radius : h - 1;
      T m = PoolBits<T>::neg_inf();
      float mv = -INFINITY;
      for (int q = q0; q <= q1; ++q) pool_update(m, mv, hmax[(q - in0) * row_elems + rest]);
      dst[e] = PoolBits<T>::finish(m);
    }
    __syncthreads();
  }
}

// SPPF: per (image, channel block) plane held whole in shared memory, with a
// 2-pixel -inf border so every 5-wide window is full (-inf never wins under the
// CPU rule, so this equals clipping the window at the edge).  Planes without NaN
// or -0 take a half2 max (equal values then have equal bits, so any max is the
// CPU's first max); planes holding either take the exact per-lane CPU rule.
// out planes: [x, p1, p2, p3] at channel blocks cb, c1+cb, 2c1+cb, 3c1+cb.
__device__ __forceinline__ bool special_word(uint32_t w) {
  uint32_t nan = __vcmpgtu2(w & 0x7fff7fffu, 0x7c007c00u);
  uint32_t negzero = __vcmpeq2(w, 0x80008000u);
  return (nan | negzero) != 0u;
}

__device__ __forceinline__ uint4 hmax4(uint4 a, uint4 b) {
  __half2 r[4];
  const __half2* pa = reinterpret_cast<const __half2*>(&a);
  const __half2* pb = reinterpret_cast<const __half2*>(&b);
#pragma unroll
  for (int i = 0; i < 4; ++i) r[i] = __hmax2(pa[i], pb[i]);
  return *reinterpret_cast<uint4*>(r);
}

__global__ void __launch_bounds__(256) sppf_planes(const uint16_t* x, uint16_t* out, int64_t n,
                                                   int64_t c1, int h, int w, int radius) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int pw = w + 2 * radius, ph = h + 2 * radius;  // padded plane, in pixels
  const int padded_vec = ph * pw * 2;                 // uint4 per padded plane
  uint4* cur = reinterpret_cast<uint4*>(smem_raw);
  uint4* tmp = cur + padded_vec;
  const int plane_vec = h * w * 2;
  const uint4 ninf = make_uint4(0xfc00fc00u, 0xfc00fc00u, 0xfc00fc00u, 0xfc00fc00u);
  for (int v = threadIdx.x; v < 2 * padded_vec; v += blockDim.x) cur[v] = ninf;
  __syncthreads();
  for (int64_t job = blockIdx.x; job < n * c1; job += gridDim.x) {
    int64_t b = job / c1, cb = job % c1;
    const uint4* src = reinterpret_cast<const uint4*>(x + job * (int64_t)plane_vec * 8);
    uint4* dst0 = reinterpret_cast<uint4*>(out + ((b * 4 * c1) + cb) * (int64_t)plane_vec * 8);
    bool special = false;
    for (int v = threadIdx.x; v < plane_vec; v += blockDim.x) {
      uint4 q = src[v];
      dst0[v] = q;
      int pix = v >> 1, row = pix / w, col = pix % w;
      cur[((row + radius) * pw + col + radius) * 2 + (v & 1)] = q;
      special |= special_word(q.x) | special_word(q.y) | special_word(q.z) | special_word(q.w);
    }
    special = __syncthreads_or(special);
    for (int stage = 1; stage <= 3; ++stage) {
      // horizontal: tmp[row][col] over every padded row (border rows stay -inf)
      for (int v = threadIdx.x; v < plane_vec; v += blockDim.x) {
        int pix = v >> 1, row = pix / w + radius, col = pix % w + radius, j = v & 1;
        const uint4* r = cur + (row * pw + col - radius) * 2 + j;
        uint4 m;
        if (!special) {
          m = r[0];
          for (int k = 1; k <= 2 * radius; ++k) m = hmax4(m, r[2 * k]);
        } else {
          uint16_t best[8];
          float bv[8];
#pragma unroll
          for (int l = 0; l < 8; ++l) { best[l] = 0xfc00u; bv[l] = -INFINITY; }
          for (int k = 0; k <= 2 * radius; ++k) {
            uint4 q = r[2 * k];
            const uint16_t* e = reinterpret_cast<const uint16_t*>(&q);
#pragma unroll
            for (int l = 0; l < 8; ++l) pool_update(best[l], bv[l], e[l]);
          }
          m = *reinterpret_cast<uint4*>(best);
        }
        tmp[(row * pw + col) * 2 + j] = m;
      }
      __syncthreads();
      uint4* dst = reinterpret_cast<uint4*>(out + ((b * 4 * c1) + stage * c1 + cb) * (int64_t)plane_vec * 8);
      for (int v = threadIdx.x; v < plane_vec; v += blockDim.x) {
        int pix = v >> 1, row = pix / w + radius, col = pix % w + radius, j = v & 1;
        const uint4* r = tmp + ((row - radius) * pw + col) * 2 + j;
        uint4 m;
        if (!special) {
          m = r[0];
          for (int k = 1; k <= 2 * radius; ++k) m = hmax4(m, r[2 * k * pw]);
        } else {
          uint16_t best[8];
          float bv[8];
#pragma unroll
          for (int l = 0; l < 8; ++l) { best[l] = 0xfc00u; bv[l] = -INFINITY; }
          for (int k = 0; k <= 2 * radius; ++k) {
            uint4 q = r[2 * k * pw];
            const uint16_t* e = reinterpret_cast<const uint16_t*>(&q);
#pragma unroll
            for (int l = 0; l < 8; ++l) pool_update(best[l], bv[l], e[l]);
          }
#pragma unroll
          for (int l = 0; l < 8; ++l) best[l] = PoolBits<uint16_t>::finish(best[l]);
          m = *reinterpret_cast<uint4*>(best);
        }
        cur[(row * pw + col) * 2 + j] = m;
        dst[v] = m;
      }
      __syncthreads();
    }
  }
}

// sppf_planes for planes of at most 4 * 256 16-byte vectors (e.g. the 20x20
// SPPF of a 640 model): every plane has the same geometry, so each thread
// computes the padded shared-memory position of its (at most VPT) vectors once,
// and the three stages run without any index division.
template <int VPT>
__global__ void __launch_bounds__(256) sppf_planes_small(const uint16_t* x, uint16_t* out, int64_t n,
                                                         int64_t c1, int h, int w, int radius) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int pw = w + 2 * radius, ph = h + 2 * radius;  // padded plane, in pixels
  const int padded_vec = ph * pw * 2;                 // uint4 per padded plane
  uint4* cur = reinterpret_cast<uint4*>(smem_raw);
  uint4* tmp = cur + padded_vec;
  const int plane_vec = h * w * 2;
  const uint4 ninf = make_uint4(0xfc00fc00u, 0xfc00fc00u, 0xfc00fc00u, 0xfc00fc00u);
  int pos[VPT];  // padded position of vector tid + k*256 (-1: none)
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = threadIdx.x + k * 256;
    const int pix = v >> 1, row = pix / w, col = pix - row * w;
    pos[k] = v < plane_vec ? ((row + radius) * pw + col + radius) * 2 + (v & 1) : -1;
  }
  for (int v = threadIdx.x; v < 2 * padded_vec; v += blockDim.x) cur[v] = ninf;
  __syncthreads();
  const int row_step = 2 * pw;
  for (int64_t job = blockIdx.x; job < n * c1; job += gridDim.x) {
    const int64_t b = job / c1, cb = job - b * c1;
    const uint4* src = reinterpret_cast<const uint4*>(x + job * (int64_t)plane_vec * 8);
    uint4* dst0 = reinterpret_cast<uint4*>(out + ((b * 4 * c1) + cb) * (int64_t)plane_vec * 8);
    bool special = false;
    uint4 q[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k)
      if (pos[k] >= 0) q[k] = src[threadIdx.x + k * 256];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      if (pos[k] >= 0) {
        dst0[threadIdx.x + k * 256] = q[k];
        cur[pos[k]] = q[k];
        special |= special_word(q[k].x) | special_word(q[k].y) | special_word(q[k].z) | special_word(q[k].w);
      }
    }
    special = __syncthreads_or(special);
    for (int stage = 1; stage <= 3; ++stage) {
#pragma unroll
      for (int k = 0; k < VPT; ++k) {  // horizontal: tmp[row][col] (border rows stay -inf)
        if (pos[k] < 0) continue;
        const uint4* r = cur + pos[k] - 2 * radius;
        uint4 m;
        if (!special) {
          m = r[0];
          for (int t = 1; t <= 2 * radius; ++t) m = hmax4(m, r[2 * t]);
        } else {
          uint16_t best[8];
          float bv[8];
#pragma unroll
          for (int l = 0; l < 8; ++l) { best[l] = 0xfc00u; bv[l] = -INFINITY; }
          for (int t = 0; t <= 2 * radius; ++t) {
            uint4 e4 = r[2 * t];
            const uint16_t* e = reinterpret_cast<const uint16_t*>(&e4);
#pragma unroll
            for (int l = 0; l < 8; ++l) pool_update(best[l], bv[l], e[l]);
          }
          m = *reinterpret_cast<uint4*>(best);
        }
        tmp[pos[k]] = m;
      }
      __syncthreads();
      uint4* dst = reinterpret_cast<uint4*>(out + ((b * 4 * c1) + stage * c1 + cb) * (int64_t)plane_vec * 8);
#pragma unroll
      for (int k = 0; k < VPT; ++k) {  // vertical, into cur and the stage's output slice
        if (pos[k] < 0) continue;
        const uint4* r = tmp + pos[k] - radius * row_step;
        uint4 m;
        if (!special) {
          m = r[0];
          for (int t = 1; t <= 2 * radius; ++t) m = hmax4(m, r[t * row_step]);
        } else {
          uint16_t best[8];
          float bv[8];
#pragma unroll
          for (int l = 0; l < 8; ++l) { best[l] = 0xfc00u; bv[l] = -INFINITY; }
          for (int t = 0; t <= 2 * radius; ++t) {
            uint4 e4 = r[t * row_step];
            const uint16_t* e = reinterpret_cast<const uint16_t*>(&e4);
#pragma unroll
            for (int l = 0; l < 8; ++l) pool_update(best[l], bv[l], e[l]);
          }
#pragma unroll
          for (int l = 0; l < 8; ++l) best[l] = PoolBits<uint16_t>::finish(best[l]);
          m = *reinterpret_cast<uint4*>(best);
        }
        cur[pos[k]] = m;
        dst[threadIdx.x + k * 256] = m;
      }
      __syncthreads();
    }
  }
}

// SPPF with a 5x5 window (radius 2), the YOLO case, in runs of four outputs:
// each thread of the horizontal pass takes a run of four output pixels of one row
// (and one half of the 16 channel lanes), loads the eight-pixel window once and
// shares the partial maxima between the four outputs; the vertical pass does the
// same along a column.  So a pool stage costs two shared-memory loads and one
// store per output vector and pass, instead of five loads.  Planes whose width
// and height are rounded up to multiples of 4 sit in shared memory with a 2-pixel
// -inf border (padded columns and rows past the image stay -inf).  Planes with a
// NaN or -0 take the CPU's exact per-lane rule over the same windows.
__device__ __forceinline__ void run_max4(const uint4 (&x)[8], uint4 (&y)[4]) {
  const uint4 c34 = hmax4(x[3], x[4]), a12 = hmax4(x[1], x[2]), b56 = hmax4(x[5], x[6]);
  y[0] = hmax4(hmax4(x[0], a12), c34);
  y[1] = hmax4(a12, hmax4(c34, x[5]));
  y[2] = hmax4(hmax4(x[2], c34), b56);
  y[3] = hmax4(c34, hmax4(b56, x[7]));
}

// A whole plane under the CPU's exact per-lane rule (planes holding NaN or -0;
// the CTA branches here together): three chained 5x5 pools, each a horizontal
// pass cur -> tmp and a vertical pass tmp -> cur and the stage's output slice,
// every window folded in index order (first maximum, last NaN, NaN quieted on
// the vertical pass).  Out of line so the fast path's registers stay its own.
__device__ __noinline__ void sppf_plane_exact(uint4* cur, uint4* tmp, int pw, int h, int w, uint4* const* dst) {
  auto at = [&](int prow, int pcol, int hf) { return (prow * pw + (pcol ^ ((pcol >> 2) & 3))) * 2 + hf; };
  const int plane_vec = h * w * 2;
  for (int stage = 0; stage < 3; ++stage) {
    for (int pass = 0; pass < 2; ++pass) {
      for (int v = threadIdx.x; v < plane_vec; v += blockDim.x) {
        const int pix = v >> 1, row = pix / w, col = pix - row * w, hf = v & 1;
        uint16_t best[8];
        float bv[8];
#pragma unroll
        for (int l = 0; l < 8; ++l) {
          best[l] = 0xfc00u;
          bv[l] = -INFINITY;
        }
        for (int t = -2; t <= 2; ++t) {
          const uint4 q = pass == 0 ? cur[at(row + 2, col + 2 + t, hf)] : tmp[at(row + 2 + t, col + 2, hf)];
          const uint16_t* e = reinterpret_cast<const uint16_t*>(&q);
#pragma unroll
          for (int l = 0; l < 8; ++l) pool_update(best[l], bv[l], e[l]);
        }
        if (pass == 1) {
#pragma unroll
          for (int l = 0; l < 8; ++l) best[l] = PoolBits<uint16_t>::finish(best[l]);
        }
        const uint4 m = *reinterpret_cast<uint4*>(best);
        if (pass == 0) {
          tmp[at(row + 2, col + 2, hf)] = m;
        } else {
          dst[stage][v] = m;
          if (stage < 2) cur[at(row + 2, col + 2, hf)] = m;
        }
      }
      __syncthreads();
    }
  }
}

// Row pitch, in pixels, of sppf_runs' padded planes: the 4-aligned width, the 2-pixel
// borders, and one or two unused columns so consecutive rows start on different
// 16-byte bank groups (a pitch of a multiple of 8 vectors put the horizontal runs of
// neighbouring rows on the same banks: a quarter of the passes' shared-memory
// wavefronts were conflict replays at 20 x 20; one column more leaves 7%).
__host__ __device__ __forceinline__ int sppf_pitch(int w) {
  const int w4 = (w + 3) & ~3;
  return w4 + 4 + (((w4 >> 2) & 1) ? 1 : 2);
}

// Each thread takes at most IPT runs per pass; every plane has the same
// geometry, so the runs' shared-memory bases and swizzle terms are computed once
// per kernel.
template <int IPT>
__global__ void __launch_bounds__(256, 4) sppf_runs(const uint16_t* x, uint16_t* out, int64_t n, int64_t c1, int h,
                                                 int w, FastDiv wdiv) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int w4 = (w + 3) & ~3, h4 = (h + 3) & ~3;
  const int pw = sppf_pitch(w), ph = h4 + 4;  // padded plane, in pixels (columns past w4 + 3 unused)
  const int padded_vec = ph * pw * 2;
  uint4* cur = reinterpret_cast<uint4*>(smem_raw);  // the plane being pooled
  uint4* tmp = cur + padded_vec;                     // the horizontal-pass scratch
  // Vector of (padded row, padded column, half): the column is XOR-swizzled inside
  // its aligned block of four by the block index, so the lanes of a horizontal run
  // pass (runs four pixels apart) spread over all eight 16-byte bank groups.
  auto at = [&](int prow, int pcol, int hf) { return (prow * pw + (pcol ^ ((pcol >> 2) & 3))) * 2 + hf; };
  const int plane_vec = h * w * 2;
  const int runs_w = w4 / 4, runs_h = h4 / 4;
  const int h_items = h * runs_w * 2, v_items = w * runs_h * 2;
  // horizontal run i: window vectors k < 4 at hb + 2 (k ^ s1), k >= 4 at hb + 8 + 2 ((k - 4) ^ s2);
  // output k (k < hvalid) at column 4q + k + 2 (k < 2 in block q, else block q + 1)
  int hb[IPT], hs[IPT], hvalid[IPT], vb[IPT], vvalid[IPT], vout[IPT];
#pragma unroll
  for (int i = 0; i < IPT; ++i) {
    const int e = threadIdx.x + i * 256;
    hvalid[i] = vvalid[i] = 0;
    hb[i] = hs[i] = vb[i] = vout[i] = 0;
    if (e < h_items) {
      const int hf = e & 1, t = e >> 1, q = t % runs_w, row = t / runs_w;
      hb[i] = ((row + 2) * pw + 4 * q) * 2 + hf;
      hs[i] = (q & 3) | (((q + 1) & 3) << 2);
      hvalid[i] = w - 4 * q < 4 ? w - 4 * q : 4;
    }
    if (e < v_items) {
      const int hf = e & 1, t = e >> 1, col = t % w, q = t / w;
      vb[i] = at(4 * q, col + 2, hf);
      vout[i] = ((4 * q) * w + col) * 2 + hf;
      vvalid[i] = h - 4 * q < 4 ? h - 4 * q : 4;
    }
  }
  const int row_step = 2 * pw;
  const uint4 ninf = make_uint4(0xfc00fc00u, 0xfc00fc00u, 0xfc00fc00u, 0xfc00fc00u);
  for (int v = threadIdx.x; v < 2 * padded_vec; v += blockDim.x) cur[v] = ninf;
  pdl_trigger();
  pdl_wait();
  __syncthreads();
#pragma unroll 1
  for (int64_t job = blockIdx.x; job < n * c1; job += gridDim.x) {
    const int64_t b = job / c1, cb = job - b * c1;
    const uint4* src = reinterpret_cast<const uint4*>(x + job * (int64_t)plane_vec * 8);
    uint4* dst0 = reinterpret_cast<uint4*>(out + ((b * 4 * c1) + cb) * (int64_t)plane_vec * 8);
    bool special = false;
    for (int v = threadIdx.x; v < plane_vec; v += blockDim.x) {  // slice 0 of the concat: the plane itself
      const uint4 q = src[v];
      dst0[v] = q;
      const int pix = v >> 1, row = (int)wdiv.div((uint32_t)pix), col = pix - row * w;
      cur[at(row + 2, col + 2, v & 1)] = q;
      special |= special_word(q.x) | special_word(q.y) | special_word(q.z) | special_word(q.w);
    }
    special = __syncthreads_or(special);
    uint4* const slices[3] = {
        reinterpret_cast<uint4*>(out + ((b * 4 * c1) + c1 + cb) * (int64_t)plane_vec * 8),
        reinterpret_cast<uint4*>(out + ((b * 4 * c1) + 2 * c1 + cb) * (int64_t)plane_vec * 8),
        reinterpret_cast<uint4*>(out + ((b * 4 * c1) + 3 * c1 + cb) * (int64_t)plane_vec * 8)};
    if (special) {
      sppf_plane_exact(cur, tmp, pw, h, w, slices);
    } else {
#pragma unroll 1
      for (int stage = 1; stage <= 3; ++stage) {
#pragma unroll
        for (int i = 0; i < IPT; ++i) {  // horizontal runs: cur -> tmp
          if (!hvalid[i]) continue;
          const int s1 = hs[i] & 3, s2 = hs[i] >> 2, base = hb[i];
          uint4 xs[8], ys[4];
#pragma unroll
          for (int k = 0; k < 8; ++k) xs[k] = cur[base + (k < 4 ? 2 * (k ^ s1) : 8 + 2 * ((k - 4) ^ s2))];
          run_max4(xs, ys);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (k < hvalid[i]) tmp[base + (k < 2 ? 2 * ((k + 2) ^ s1) : 8 + 2 * ((k - 2) ^ s2))] = ys[k];
        }
        __syncthreads();
        uint4* dst = slices[stage - 1];
        const bool keep = stage < 3;  // the last stage's result only goes to the output
#pragma unroll
        for (int i = 0; i < IPT; ++i) {  // vertical runs: tmp -> cur and the output
          if (!vvalid[i]) continue;
          const int base = vb[i];
          uint4* og = dst + vout[i];
          uint4 xs[8], ys[4];
#pragma unroll
          for (int k = 0; k < 8; ++k) xs[k] = tmp[base + k * row_step];
          run_max4(xs, ys);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (k < vvalid[i]) {
              if (keep) cur[base + (k + 2) * row_step] = ys[k];
              og[2 * k * w] = ys[k];
            }
          }
        }
        __syncthreads();
      }
    }
  }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }


}  // namespace
}  // namespace ttn

using namespace ttn;

extern "C" {

ttn_status ttn_nc1hwc0_to_nchw_f16(const void* x, int64_t n, int64_t c1, int64_t hw,
                                   int64_t channels, void* y, int64_t y_batch_stride,
                                   int64_t y_channel_stride, ttn_stream stream) {
  const char* name = "ttn_nc1hwc0_to_nchw_f16";
  if (n < 0 || c1 < 0 || hw < 0 || channels < 0 || channels > c1 * 16)
    return fail(TTN_INVALID_ARG, "%s: bad sizes", name);
  if (!n || !c1 || !hw || !channels) return TTN_OK;
  if (!x || !y) return fail(TTN_INVALID_ARG, "%s: null pointer", name);
  if (!aligned16(x)) return fail(TTN_INVALID_ARG, "%s: x must be 16-byte aligned", name);
  if (((uintptr_t)y & 1u)) return fail(TTN_INVALID_ARG, "%s: y not 2-byte aligned", name);
  bool vec = aligned16(y) && y_batch_stride % 8 == 0 && y_channel_stride % 8 == 0;
  if (((uintptr_t)y & 7u) == 0 && y_batch_stride % 4 == 0 && y_channel_stride % 4 == 0 && hw % 4 == 0) {
    int64_t threads = n * c1 * (hw / 4);
    TTN_TRY(cuda_check(launch_pdl(blocked_to_nchw_regs, dim3(grid_for(threads, 256, 8)), dim3(256), 0,
                                  (cudaStream_t)stream, (const uint4*)x, n, c1, hw,
                                  (c1 * 16 < channels ? c1 * 16 : channels), (uint16_t*)y, y_batch_stride,
                                  y_channel_stride),
                       name));
    return launch_check(name);
  }
  int64_t jobs = n * c1 * ((hw + kPix - 1) / kPix);
  unsigned grid = (unsigned)(jobs < (int64_t)sm_count() * 16 ? jobs : (int64_t)sm_count() * 16);
  blocked_to_nchw<<<grid, 128, 0, (cudaStream_t)stream>>>(
      (const uint16_t*)x, n, c1, hw, (c1 * 16 < channels ? c1 * 16 : channels), (uint16_t*)y,
      y_batch_stride, y_channel_stride, vec);
  return launch_check(name);
}

ttn_status ttn_nchw_to_nc1hwc0_f16(const void* x, int64_t n, int64_t channels, int64_t hw,
                                   void* y, ttn_stream stream) {
  const char* name = "ttn_nchw_to_nc1hwc0_f16";
  if (n < 0 || channels < 0 || hw < 0) return fail(TTN_INVALID_ARG, "%s: bad sizes", name);
  if (!n || !channels || !hw) return TTN_OK;
  if (!x || !y) return fail(TTN_INVALID_ARG, "%s: null pointer", name);
  if (!aligned16(y)) return fail(TTN_INVALID_ARG, "%s: y must be 16-byte aligned", name);
  if (((uintptr_t)x & 1u)) return fail(TTN_INVALID_ARG, "%s: x not 2-byte aligned", name);
  bool vec = aligned16(x) && hw % 8 == 0;
  int64_t jobs = n * ((channels + 15) / 16) * ((hw + kPix - 1) / kPix);
  unsigned grid = (unsigned)(jobs < (int64_t)sm_count() * 16 ? jobs : (int64_t)sm_count() * 16);
  nchw_to_blocked<<<grid, 128, 0, (cudaStream_t)stream>>>((const uint16_t*)x, n, channels, hw,
                                                          (uint16_t*)y, vec);
  return launch_check(name);
}

ttn_status ttn_upsample2x(int layout, int dtype, const void* x, void* y, int64_t n, int64_t c,
                          int64_t h, int64_t w, ttn_stream stream) {
  const char* name = "ttn_upsample2x";
  if (layout != TTN_NCHW && layout != TTN_NC1HWC0) return fail(TTN_INVALID_ARG, "%s: layout", name);
  if (dtype != TTN_F16 && dtype != TTN_F32) return fail(TTN_UNSUPPORTED, "%s: dtype", name);
  if (n < 0 || c < 0 || h < 0 || w < 0) return fail(TTN_INVALID_ARG, "%s: negative size", name);
  if (!n || !c || !h || !w) return TTN_OK;
  if (!x || !y) return fail(TTN_INVALID_ARG, "%s: null pointer", name);
  cudaStream_t s = (cudaStream_t)stream;
  if (layout == TTN_NC1HWC0) {
    if (dtype != TTN_F16) return fail(TTN_UNSUPPORTED, "%s: NC1HWC0 supports float16", name);
    if (!aligned16(x) || !aligned16(y)) return fail(TTN_INVALID_ARG, "%s: 16-byte alignment", name);
    int64_t nvec = n * c * h * w * 2;
    if (nvec < ((int64_t)1 << 31))
      upsample_blocked32<<<grid_for(nvec, 256), 256, 0, s>>>(
          (const uint4*)x, (uint4*)y, (uint32_t)nvec, FastDiv((uint32_t)(c * h * w * 2)), FastDiv((uint32_t)h),
          FastDiv((uint32_t)w), c * h * w * 2, c * h * w * 8);
    else
      upsample_blocked<<<grid_for(nvec, 256), 256, 0, s>>>((const uint4*)x, (uint4*)y, n, c, h, w,
                                                           c * h * w * 2, c * h * w * 8);
    return launch_check(name);
  }
  if (dtype == TTN_F16 && w % 4 == 0 && aligned16(y) && ((uintptr_t)x & 7u) == 0) {
    int64_t nvec = n * c * h * (w / 4);
    upsample_nchw_vec<<<grid_for(nvec, 256), 256, 0, s>>>((const uint2*)x, (uint4*)y, n * c, h,
                                                          w / 4);
  } else if (dtype == TTN_F16) {
    upsample_nchw_scalar<uint16_t><<<grid_for(n * c * h * w * 4, 256), 256, 0, s>>>(
        (const uint16_t*)x, (uint16_t*)y, n * c, h, w);
  } else {
    upsample_nchw_scalar<uint32_t><<<grid_for(n * c * h * w * 4, 256), 256, 0, s>>>(
        (const uint32_t*)x, (uint32_t*)y, n * c, h, w);
  }
  return launch_check(name);
}

ttn_status ttn_upsample2x_nc1hwc0_f16(const void* x, int64_t x_batch_stride, void* y,
                                      int64_t y_batch_stride, int64_t n, int64_t c1, int64_t h,
                                      int64_t w, ttn_stream stream) {
  const char* name = "ttn_upsample2x_nc1hwc0_f16";
  if (n < 0 || c1 < 0 || h < 0 || w < 0) return fail(TTN_INVALID_ARG, "%s: negative size", name);
  if (!n || !c1 || !h || !w) return TTN_OK;
  if (!x || !y) return fail(TTN_INVALID_ARG, "%s: null pointer", name);
  if (!aligned16(x) || !aligned16(y) || x_batch_stride % 8 || y_batch_stride % 8)
    return fail(TTN_INVALID_ARG, "%s: pointers and batch strides must be 16-byte multiples", name);
  if (x_batch_stride < c1 * h * w * 16 || y_batch_stride < c1 * h * w * 64)
    return fail(TTN_INVALID_ARG, "%s: batch stride smaller than one image", name);
  int64_t nvec = n * c1 * h * w * 2;
  if (nvec < ((int64_t)1 << 31)) {
    TTN_TRY(cuda_check(launch_pdl(upsample_blocked32, dim3(grid_for(nvec, 256)), dim3(256), 0, (cudaStream_t)stream,
                                  (const uint4*)x, (uint4*)y, (uint32_t)nvec, FastDiv((uint32_t)(c1 * h * w * 2)),
                                  FastDiv((uint32_t)h), FastDiv((uint32_t)w), x_batch_stride / 8,
                                  y_batch_stride / 8),
                       name));
    return launch_check(name);
  }
  upsample_blocked<<<grid_for(nvec, 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint4*)x, (uint4*)y, n, c1, h, w, x_batch_stride / 8, y_batch_stride / 8);
  return launch_check(name);
}

ttn_status ttn_maxpool(int layout, int dtype, int32_t kernel, const void* x, void* y, int64_t n,
                       int64_t c, int64_t h, int64_t w, ttn_stream stream) {
  const char* name = "ttn_maxpool";
  if (layout != TTN_NCHW && layout != TTN_NC1HWC0) return fail(TTN_INVALID_ARG, "%s: layout", name);
  if (dtype != TTN_F16 && dtype != TTN_F32) return fail(TTN_UNSUPPORTED, "%s: dtype", name);
  if (kernel < 1 || kernel % 2 == 0)
    return fail(TTN_INVALID_ARG, "%s: maxpool kernel must be a positive odd integer", name);
  if (n < 0 || c < 0 || h < 0 || w < 0) return fail(TTN_INVALID_ARG, "%s: negative size", name);
  if (!n || !c || !h || !w) return TTN_OK;
  if (!x || !y) return fail(TTN_INVALID_ARG, "%s: null pointer", name);
  if (h > (1 << 20) || w > (1 << 20)) return fail(TTN_UNSUPPORTED, "%s: plane too large", name);
  if (layout == TTN_NC1HWC0 && dtype != TTN_F16)
    return fail(TTN_UNSUPPORTED, "%s: NC1HWC0 supports float16", name);
  const int lanes = layout == TTN_NC1HWC0 ? 16 : 1;
  const int radius = kernel / 2;
  const size_t es = dtype_size(dtype);
  const size_t row_bytes = (size_t)w * lanes * es;
  const int limit = max_dynamic_smem();
  // band rows: as many as fit two staged copies of (band + 2r) rows
  int64_t band = (int64_t)(limit / (2 * row_bytes)) - 2 * radius;
  if (band < 1) return fail(TTN_UNSUPPORTED, "%s: a row band exceeds shared memory", name);
  int64_t want = (int64_t)(8192 / (w * lanes)) + 1;  // ~8K outputs per block
  if (band > want) band = want;
  if (band > h) band = h;
  size_t smem = 2 * (size_t)(band + 2 * radius) * row_bytes;
  int64_t planes = layout == TTN_NC1HWC0 ? n * c : n * c;
  int64_t jobs = planes * ((h + band - 1) / band);
  unsigned grid = (unsigned)(jobs < (int64_t)sm_count() * 8 ? jobs : (int64_t)sm_count() * 8);
  cudaStream_t s = (cudaStream_t)stream;
  if (es == 2) {
    TTN_TRY(ensure_dynamic_smem((const void*)maxpool_band<uint16_t>, (int)smem));
    maxpool_band<uint16_t><<<grid, 256, smem, s>>>((const uint16_t*)x, (uint16_t*)y, planes, (int)h,
                                                   (int)w, lanes, radius, (int)band);
  } else {
    TTN_TRY(ensure_dynamic_smem((const void*)maxpool_band<uint32_t>, (int)smem));
    maxpool_band<uint32_t><<<grid, 256, smem, s>>>((const uint32_t*)x, (uint32_t*)y, planes, (int)h,
                                                   (int)w, lanes, radius, (int)band);
  }
  return launch_check(name);
}

ttn_status ttn_sppf_f16(const void* x, void* out, int64_t n, int64_t c1, int64_t h, int64_t w,
                        int32_t kernel, ttn_stream stream) {
  const char* name = "ttn_sppf_f16";
  if (kernel < 1 || kernel % 2 == 0)
    return fail(TTN_INVALID_ARG, "%s: kernel must be a positive odd integer", name);
  if (n < 0 || c1 < 0 || h < 0 || w < 0) return fail(TTN_INVALID_ARG, "%s: negative size", name);
  if (!n || !c1 || !h || !w) return TTN_OK;
  if (!x || !out) return fail(TTN_INVALID_ARG, "%s: null pointer", name);
  if (!aligned16(x) || !aligned16(out)) return fail(TTN_INVALID_ARG, "%s: 16-byte alignment", name);
  const int64_t r = kernel / 2;
  size_t smem = 2 * (size_t)(h + 2 * r) * (w + 2 * r) * 16 * 2;
  cudaStream_t s = (cudaStream_t)stream;
  if ((int64_t)smem > max_dynamic_smem()) {
    // Plane too large to hold twice: three chained pools through the output.
    const int64_t plane = h * w * 16;
    TTN_TRY(cuda_check(cudaMemcpy2DAsync(out, 4 * c1 * plane * 2, x, c1 * plane * 2, c1 * plane * 2,
                                         n, cudaMemcpyDeviceToDevice, s),
                       name));
    for (int stage = 1; stage <= 3; ++stage) {
      // pool each image's previous stage slice into the next slice
      for (int64_t b = 0; b < n; ++b) {
        const uint16_t* src = (const uint16_t*)out + (b * 4 * c1 + (stage - 1) * c1) * plane;
        uint16_t* dst = (uint16_t*)out + (b * 4 * c1 + stage * c1) * plane;
        TTN_TRY(ttn_maxpool(TTN_NC1HWC0, TTN_F16, kernel, src, dst, 1, c1, h, w, stream));
      }
    }
    return TTN_OK;
  }
  int64_t jobs = n * c1;
  const int64_t plane_vec = h * w * 2;
  const size_t runs_smem = 2 * (size_t)(((h + 3) & ~3) + 4) * sppf_pitch((int)w) * 16 * 2;
  const int64_t runs = h * ((w + 3) / 4) * 2 > w * ((h + 3) / 4) * 2 ? h * ((w + 3) / 4) * 2 : w * ((h + 3) / 4) * 2;
  if (kernel == 5 && runs <= 2 * 256 && (int64_t)runs_smem <= max_dynamic_smem()) {
    // the YOLO window: runs of four, fixed per-thread geometry
    const void* fn = runs <= 256 ? (const void*)sppf_runs<1> : (const void*)sppf_runs<2>;
    TTN_TRY(ensure_dynamic_smem(fn, (int)runs_smem));
    unsigned grid = resident_grid(fn, 256, runs_smem, jobs, 1);
    if (runs <= 256)
      TTN_TRY(cuda_check(launch_pdl(sppf_runs<1>, dim3(grid), dim3(256), runs_smem, s, (const uint16_t*)x,
                                    (uint16_t*)out, n, c1, (int)h, (int)w, FastDiv((uint32_t)w)),
                         name));
    else
      TTN_TRY(cuda_check(launch_pdl(sppf_runs<2>, dim3(grid), dim3(256), runs_smem, s, (const uint16_t*)x,
                                    (uint16_t*)out, n, c1, (int)h, (int)w, FastDiv((uint32_t)w)),
                         name));
    return launch_check(name);
  }
  if (plane_vec <= 4 * 256) {  // fixed per-thread positions
    const int vpt = (int)((plane_vec + 255) / 256);
    const void* fn = vpt == 1 ? (const void*)sppf_planes_small<1>
                   : vpt == 2 ? (const void*)sppf_planes_small<2>
                   : vpt == 3 ? (const void*)sppf_planes_small<3>
                              : (const void*)sppf_planes_small<4>;
    TTN_TRY(ensure_dynamic_smem(fn, (int)smem));
    unsigned grid = resident_grid(fn, 256, smem, jobs, 1);
    if (vpt == 1)
      sppf_planes_small<1><<<grid, 256, smem, s>>>((const uint16_t*)x, (uint16_t*)out, n, c1, (int)h, (int)w, (int)r);
    else if (vpt == 2)
      sppf_planes_small<2><<<grid, 256, smem, s>>>((const uint16_t*)x, (uint16_t*)out, n, c1, (int)h, (int)w, (int)r);
    else if (vpt == 3)
      sppf_planes_small<3><<<grid, 256, smem, s>>>((const uint16_t*)x, (uint16_t*)out, n, c1, (int)h, (int)w, (int)r);
    else
      sppf_planes_small<4><<<grid, 256, smem, s>>>((const uint16_t*)x, (uint16_t*)out, n, c1, (int)h, (int)w, (int)r);
    return launch_check(name);
  }
  TTN_TRY(ensure_dynamic_smem((const void*)sppf_planes, (int)smem));
  int per_sm = (int)(200 * 1024 / (smem ? smem : 1));
  if (per_sm < 1) per_sm = 1;
  unsigned grid = (unsigned)(jobs < (int64_t)sm_count() * per_sm ? jobs : (int64_t)sm_count() * per_sm);
  sppf_planes<<<grid, 256, smem, s>>>((const uint16_t*)x, (uint16_t*)out, n, c1, (int)h, (int)w,
                                      kernel / 2);
  return launch_check(name);
}

}  // extern "C"
