// Depthwise 2-D convolution over NC1HWC0 fp16 (the YOLO11 head's DWConv), with the
// reference's fused epilogue (depthwise_kernel depthwise_flow.cpp:23-162):
//   acc = 0; for ky, for kx: acc = acc + x * w   (FP32, product and sum each rounded)
//   acc = acc + bias;  y = fp16(acc / (1 + exp(-acc)))  (or fp16(acc) unfused).
// The taps are taken in the reference's order.  x and w are fp16 values, so every
// product x * w (11 x 11 significant bits) is exact in FP32 and the reference's
// rounded product followed by a rounded sum is one correctly rounded fused
// multiply-add: the unfused result is bit-identical to the reference's.  The SiLU
// differs only by the exp of the two libraries.
//
// HBM-bound CUDA-core work, kept under the issue limit.  One CTA per (image, channel
// block, band of output rows): the band's input rows, with a zero border, are staged
// in shared memory by cp.async (zero fill for the border) as two planes of 8-channel
// 16-byte vectors; the block's k*k*16 weights and 16 biases as FP32.  A warp works on
// one plane, each thread on kDwRun adjacent output pixels of one row: it streams the
// run's input window through registers once per kernel row and applies every tap to
// every pixel it reaches, two channels per f32x2 fused multiply-add.  A run of 3
// pixels makes the lanes of a quarter warp read 48 bytes apart, 8 distinct banks.
#include <algorithm>

#include "common.cuh"

namespace ttn {
namespace {

constexpr int kDwThreads = 256;
constexpr int kDwMaxKernel = 7;
constexpr int kDwRun = 3;  // output pixels per thread along a row

// Shared memory: sw [K*K][16] FP32 weights, sb [16] FP32 biases, then the input tile
// as [plane (channels 0-7 | 8-15)][rows_in][tw] 16-byte vectors.  Four CTAs per SM
// (64 registers, at most 48 KB staged): a CTA's staging wait hides behind the other
// three's work (3 CTAs at 77 registers measured 5% slower; 5 and 6 spill).
template <int K, int S>
__global__ void __launch_bounds__(kDwThreads, 4) depthwise_nc1hwc0(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ wts, const uint16_t* __restrict__ bias,
    uint16_t* __restrict__ y, int h, int w, int oh, int ow, int band, int tw, FastDiv runs, int64_t x_bs,
    int64_t y_bs, int silu) {
  constexpr int kPad = K / 2, kSpan = (kDwRun - 1) * S + K;  // input columns a run reads per row
  extern __shared__ __align__(16) unsigned char smem[];
  const int rows_in = (band - 1) * S + K, plane = rows_in * tw;
  float* sw = reinterpret_cast<float*>(smem);
  float* sb = sw + K * K * 16;
  uint4* tile = reinterpret_cast<uint4*>(sb + 16);
  const int r0 = blockIdx.x * band, cb = blockIdx.y, img = blockIdx.z;
  const uint16_t* xin = x + img * x_bs + (int64_t)cb * h * w * 16;
  uint16_t* yout = y + img * y_bs + (int64_t)cb * oh * ow * 16;
  for (int i = threadIdx.x; i < K * K * 16; i += blockDim.x)
    sw[i] = __half2float(__ushort_as_half(wts[(int64_t)cb * K * K * 16 + i]));
  if (threadIdx.x < 16) sb[threadIdx.x] = bias ? __half2float(__ushort_as_half(bias[cb * 16 + threadIdx.x])) : 0.0f;
  const int top = r0 * S - kPad;  // input row of tile row 0
  const uint32_t tile_s = (uint32_t)__cvta_generic_to_shared(tile);
  // staging: thread = (tile column, half), walking down the rows; all copies in flight,
  // the zero border by zero-size sources
  for (int c = threadIdx.x; c < 2 * tw; c += blockDim.x) {
    const int half = c & 1, tc = c >> 1, ic = tc - kPad;
    const bool col_in = ic >= 0 && ic < w;
    const uint16_t* src = xin + ((int64_t)top * w + ic) * 16 + half * 8;
    uint32_t dst = tile_s + 16u * (half * plane + tc);
    for (int ir = top; ir < top + rows_in; ++ir, src += (int64_t)w * 16, dst += 16u * tw) {
      const bool inside = col_in && ir >= 0 && ir < h;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(inside ? src : xin),
                   "r"(inside ? 16 : 0)
                   : "memory");
    }
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  const int rows = min(band, oh - r0), units = rows * (int)runs.d;
  // item i: lane (i & 31) of a 32-run slice, plane ((i >> 5) & 1), slice (i >> 6)
  for (int i = threadIdx.x; i < ((units + 31) & ~31) * 2; i += blockDim.x) {
    const int half = (i >> 5) & 1, u = ((i >> 6) << 5) | (i & 31);
    if (u >= units) continue;
    const int lr = (int)runs.div((uint32_t)u), ox0 = (u - lr * (int)runs.d) * kDwRun;
    const unsigned long long* wq = reinterpret_cast<const unsigned long long*>(sw) + half * 4;
    const uint4* src = tile + half * plane + lr * S * tw + ox0 * S;
    unsigned long long acc[kDwRun][4];
#pragma unroll
    for (int r = 0; r < kDwRun; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[r][c] = 0ull;
#pragma unroll
    for (int ky = 0; ky < K; ++ky) {
      unsigned long long wk[K][4];
#pragma unroll
      for (int kx = 0; kx < K; ++kx) {
        const ulonglong2 a = reinterpret_cast<const ulonglong2*>(wq + (ky * K + kx) * 8)[0];
        const ulonglong2 b = reinterpret_cast<const ulonglong2*>(wq + (ky * K + kx) * 8)[1];
        wk[kx][0] = a.x, wk[kx][1] = a.y, wk[kx][2] = b.x, wk[kx][3] = b.y;
      }
#pragma unroll
      for (int j = 0; j < kSpan; ++j) {
        const uint4 v = src[ky * tw + j];
        const uint32_t words[4] = {v.x, v.y, v.z, v.w};
        unsigned long long xv[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&words[c]));
          xv[c] = f2_pack(f.x, f.y);
        }
#pragma unroll
        for (int r = 0; r < kDwRun; ++r) {
          const int kx = j - r * S;
          if (kx >= 0 && kx < K) {
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[r][c] = f2_fma(xv[c], wk[kx][c], acc[r][c]);
          }
        }
      }
    }
    const ulonglong2 b01 = reinterpret_cast<const ulonglong2*>(sb + half * 8)[0];
    const ulonglong2 b23 = reinterpret_cast<const ulonglong2*>(sb + half * 8)[1];
    const unsigned long long bq[4] = {b01.x, b01.y, b23.x, b23.y};
    uint32_t out[kDwRun][4];
#pragma unroll
    for (int r = 0; r < kDwRun; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[r][c] = f2_add(acc[r][c], bq[c]);
    if (silu) {
      // every fast pair first (independent chains the scheduler can interleave),
      // then one rarely taken branch for the lanes the bracket could not settle
      uint32_t lower[kDwRun][4], open = 0;
#pragma unroll
      for (int r = 0; r < kDwRun; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          out[r][c] = silu_pair_fast(acc[r][c], lower[r][c]);
          open |= out[r][c] ^ lower[r][c];
        }
      if (open) {
#pragma unroll
        for (int r = 0; r < kDwRun; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float2 a = f2_unpack(acc[r][c]);
            const uint32_t diff = out[r][c] ^ lower[r][c];
            if (diff & 0xffffu)
              out[r][c] = (out[r][c] & 0xffff0000u) | __half_as_ushort(__float2half_rn(silu_f32(a.x)));
            if (diff >> 16)
              out[r][c] = (out[r][c] & 0x0000ffffu) | ((uint32_t)__half_as_ushort(__float2half_rn(silu_f32(a.y))) << 16);
          }
      }
    } else {
#pragma unroll
      for (int r = 0; r < kDwRun; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float2 a = f2_unpack(acc[r][c]);
          const __half2 hv = __floats2half2_rn(a.x, a.y);
          out[r][c] = *reinterpret_cast<const uint32_t*>(&hv);
        }
    }
#pragma unroll
    for (int r = 0; r < kDwRun; ++r) {
      if (ox0 + r >= ow) break;
      reinterpret_cast<uint4*>(yout + ((int64_t)(r0 + lr) * ow + ox0 + r) * 16)[half] =
          make_uint4(out[r][0], out[r][1], out[r][2], out[r][3]);
    }
  }
}

using DwKernel = void (*)(const uint16_t*, const uint16_t*, const uint16_t*, uint16_t*, int, int, int, int, int,
                         int, FastDiv, int64_t, int64_t, int);

DwKernel depthwise_kernel(int k, int s) {
  switch (k * 4 + s) {
    case 1 * 4 + 1: return depthwise_nc1hwc0<1, 1>;
    case 1 * 4 + 2: return depthwise_nc1hwc0<1, 2>;
    case 3 * 4 + 1: return depthwise_nc1hwc0<3, 1>;
    case 3 * 4 + 2: return depthwise_nc1hwc0<3, 2>;
    case 5 * 4 + 1: return depthwise_nc1hwc0<5, 1>;
    case 5 * 4 + 2: return depthwise_nc1hwc0<5, 2>;
    case 7 * 4 + 1: return depthwise_nc1hwc0<7, 1>;
    case 7 * 4 + 2: return depthwise_nc1hwc0<7, 2>;
    default: return nullptr;
  }
}

}  // namespace
}  // namespace ttn

using namespace ttn;

extern "C" {

ttn_status ttn_depthwise_nc1hwc0_f16(const void* x, int64_t batch, int64_t c1, int64_t h, int64_t w,
                                     int64_t x_batch_stride, const void* packed_weights, const void* bias,
                                     int32_t kernel, int32_t stride, uint32_t flags, void* out,
                                     int64_t out_batch_stride, ttn_stream stream) {
  const char* name = "ttn_depthwise_nc1hwc0_f16";
  if (flags & ~TTN_CONV_SILU) return fail(TTN_INVALID_ARG, "%s: unknown flags %u", name, flags);
  if (batch < 0 || c1 <= 0 || h <= 0 || w <= 0) return fail(TTN_INVALID_ARG, "%s: sizes must be positive", name);
  if (kernel < 1 || kernel % 2 == 0 || kernel > kDwMaxKernel || (stride != 1 && stride != 2))
    return fail(TTN_UNSUPPORTED, "%s: odd kernel 1..7, stride 1 or 2", name);
  const int pad = kernel / 2;
  const int64_t oh = (h + 2 * pad - kernel) / stride + 1, ow = (w + 2 * pad - kernel) / stride + 1;
  if (oh <= 0 || ow <= 0) return fail(TTN_INVALID_ARG, "%s: kernel exceeds the padded input", name);
  if (!batch) return TTN_OK;
  if (!x || !packed_weights || !out) return fail(TTN_INVALID_ARG, "%s: null pointer", name);
  if (((uintptr_t)x | (uintptr_t)out) & 15u || ((uintptr_t)packed_weights | (uintptr_t)bias) & 1u ||
      x_batch_stride % 8 || out_batch_stride % 8)
    return fail(TTN_INVALID_ARG, "%s: 16-byte aligned x and out, batch strides that are multiples of 8", name);
  if (batch > 65535 || c1 > 65535 || h > 65535 || w > 65535)
    return fail(TTN_UNSUPPORTED, "%s: shape beyond the supported range", name);
  const int64_t runs = (ow + kDwRun - 1) / kDwRun;
  const int64_t tw = std::max<int64_t>(w + 2 * pad, (runs * kDwRun - 1) * stride + kernel);
  const size_t fixed = (size_t)(kernel * kernel * 16 + 16) * 4;
  auto staged = [&](int64_t rows) { return fixed + (size_t)(((rows - 1) * stride + kernel) * tw) * 32; };
  // output rows per CTA: about 512 runs (1024 work items, 4 per thread), staging at
  // most 48 KB (four CTAs per SM), then evened out over the bands
  int64_t band = std::min<int64_t>((512 + runs - 1) / runs, oh);
  while (band > 1 && staged(band) > 48 * 1024) --band;
  const int64_t bands = (oh + band - 1) / band;
  band = (oh + bands - 1) / bands;
  const size_t smem = staged(band);
  if ((int64_t)smem > max_dynamic_smem()) return fail(TTN_UNSUPPORTED, "%s: rows too wide", name);
  const DwKernel fn = depthwise_kernel(kernel, stride);
  TTN_TRY(ensure_dynamic_smem((const void*)fn, (int)smem));
  const dim3 grid((unsigned)bands, (unsigned)c1, (unsigned)batch);
  fn<<<grid, kDwThreads, smem, (cudaStream_t)stream>>>(
      (const uint16_t*)x, (const uint16_t*)packed_weights, (const uint16_t*)bias, (uint16_t*)out, (int)h, (int)w,
      (int)oh, (int)ow, (int)band, (int)tw, FastDiv((uint32_t)runs), batch > 1 ? x_batch_stride : 0,
      batch > 1 ? out_batch_stride : 0, (flags & TTN_CONV_SILU) ? 1 : 0);
  return launch_check(name);
}

}  // extern "C"
