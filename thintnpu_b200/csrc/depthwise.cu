// Depthwise 2-D convolution over NC1HWC0 fp16 (the YOLO11 head's DWConv), with the
// reference's fused epilogue (depthwise_kernel depthwise_flow.cpp:23-162):
//   acc = 0; for ky, for kx: acc = acc + x * w   (FP32, product and sum each rounded)
//   acc = acc + bias;  y = fp16(acc / (1 + exp(-acc)))  (or fp16(acc) unfused).
// The products and sums are taken in the reference's order, so the unfused result is
// bit-identical to it; the SiLU differs only by the exp of the two libraries.
//
// HBM-bound CUDA-core work.  One CTA per (image, channel block, band of output rows):
// the band's input rows, with a zero border of `pad` pixels, are staged in shared
// memory as fp16 16-channel vectors; the block's k*k*16 weights and 16 biases as FP32.
// The band is staged with cp.async (all copies in flight; the border by zero fill).
// Thread = (output pixel, 8 channels): k*k 16-byte shared-memory reads, one 16-byte
// store.  Bands are sized so a CTA stages at most ~48 KB.
#include "common.cuh"

namespace ttn {
namespace {

constexpr int kDwThreads = 256;
constexpr int kDwMaxKernel = 7;


__global__ void __launch_bounds__(kDwThreads) depthwise_nc1hwc0(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ wts, const uint16_t* __restrict__ bias,
    uint16_t* __restrict__ y, int c1n, int h, int w, int k, int s, int pad, int oh, int ow, int band,
    int64_t x_bs, int64_t y_bs, int silu) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int rows_in = (band - 1) * s + k, wp = w + 2 * pad;
  float* sw = reinterpret_cast<float*>(smem);                 // [k*k][16]
  float* sb = sw + k * k * 16;                                // [16]
  uint4* tile = reinterpret_cast<uint4*>(sb + 16);            // [rows_in][wp][2] (8 channels per uint4)
  const int r0 = blockIdx.x * band, cb = blockIdx.y, img = blockIdx.z;
  const uint16_t* xin = x + img * x_bs + (int64_t)cb * h * w * 16;
  uint16_t* yout = y + img * y_bs + (int64_t)cb * oh * ow * 16;
  for (int i = threadIdx.x; i < k * k * 16; i += blockDim.x)
    sw[i] = __half2float(__ushort_as_half(wts[(int64_t)cb * k * k * 16 + i]));
  if (threadIdx.x < 16) sb[threadIdx.x] = bias ? __half2float(__ushort_as_half(bias[cb * 16 + threadIdx.x])) : 0.0f;
  const int top = r0 * s - pad;  // input row of tile row 0
  const uint32_t tile_s = (uint32_t)__cvta_generic_to_shared(tile);
  for (int i = threadIdx.x; i < rows_in * wp * 2; i += blockDim.x) {  // all copies in flight, zero border
    const int half = i & 1, p = i >> 1, tr = p / wp, tc = p % wp;
    const int ir = top + tr, ic = tc - pad;
    const bool inside = ir >= 0 && ir < h && ic >= 0 && ic < w;
    const uint16_t* src = inside ? xin + ((int64_t)ir * w + ic) * 16 + half * 8 : xin;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(tile_s + 16u * i), "l"(src),
                 "r"(inside ? 16 : 0)
                 : "memory");
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  const int rows = min(band, oh - r0);
  for (int i = threadIdx.x; i < rows * ow * 2; i += blockDim.x) {
    const int half = i & 1, p = i >> 1, lr = p / ow, ox = p % ow;
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
    for (int ky = 0; ky < k; ++ky) {
      const uint4* row = tile + ((lr * s + ky) * wp + ox * s) * 2 + half;
      for (int kx = 0; kx < k; ++kx) {
        const uint4 v = row[kx * 2];
        const float* wv = sw + (ky * k + kx) * 16 + half * 8;
        const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&words[c]));
          acc[2 * c] = __fadd_rn(acc[2 * c], __fmul_rn(f.x, wv[2 * c]));
          acc[2 * c + 1] = __fadd_rn(acc[2 * c + 1], __fmul_rn(f.y, wv[2 * c + 1]));
        }
      }
    }
    uint32_t out[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float a0 = __fadd_rn(acc[2 * c], sb[half * 8 + 2 * c]), a1 = __fadd_rn(acc[2 * c + 1], sb[half * 8 + 2 * c + 1]);
      if (silu) a0 = silu_f32(a0), a1 = silu_f32(a1);
      const __half2 hv = __floats2half2_rn(a0, a1);
      out[c] = *reinterpret_cast<const uint32_t*>(&hv);
    }
    reinterpret_cast<uint4*>(yout + ((int64_t)(r0 + lr) * ow + ox) * 16)[half] = make_uint4(out[0], out[1], out[2], out[3]);
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
  const int64_t wp = w + 2 * pad;
  const size_t fixed = (size_t)(kernel * kernel * 16 + 16) * 4;
  // output rows per CTA: about 1024 (pixel, half) work items, staging at most ~48 KB
  int64_t band = (512 + ow - 1) / ow;
  if (band > oh) band = oh;
  while (band > 1 && fixed + (size_t)(((band - 1) * stride + kernel) * wp) * 32 > 48 * 1024) --band;
  const size_t smem = fixed + (size_t)(((band - 1) * stride + kernel) * wp) * 32;
  if ((int64_t)smem > max_dynamic_smem()) return fail(TTN_UNSUPPORTED, "%s: rows too wide", name);
  TTN_TRY(ensure_dynamic_smem((const void*)depthwise_nc1hwc0, (int)smem));
  const dim3 grid((unsigned)((oh + band - 1) / band), (unsigned)c1, (unsigned)batch);
  depthwise_nc1hwc0<<<grid, kDwThreads, smem, (cudaStream_t)stream>>>(
      (const uint16_t*)x, (const uint16_t*)packed_weights, (const uint16_t*)bias, (uint16_t*)out, (int)c1, (int)h,
      (int)w, kernel, stride, pad, (int)oh, (int)ow, (int)band, batch > 1 ? x_batch_stride : 0,
      batch > 1 ? out_batch_stride : 0, (flags & TTN_CONV_SILU) ? 1 : 0);
  return launch_check(name);
}

}  // extern "C"
