// Dense 2-D convolution on the 5th-generation tensor cores (tcgen05 + TMEM + TMA),
// NC1HWC0 fp16 in, fp16 out (NC1HWC0 or NCHW), FP32 accumulation, with the
// reference's fused epilogue: y = fp16(silu(acc + bias)) or fp16(acc + bias), the
// FP32 SiLU being s / (1 + exp(-s)) and one rounding at the end
// (convolution_native conv_flow.cpp:45-121, host conv() :594-646).
//
// Implicit GEMM: D[pixel, co] = sum over (tap, ci) of x[pixel shifted by tap, ci] *
// w[co, ci, tap].  A tile is 128 output pixels (a wt x ht rectangle of one image,
// wt = gcd(ow, 128)) by up to 256 output channels; K runs over (tap, group of up
// to 4 16-channel blocks), 16 channels per tcgen05.mma.  Persistent CTAs, one per
// SM, warp-specialised.  When a tile has at most 128 output channels it covers two
// 128-pixel sub-tiles (the next ht rows) that share every weight stage, halving the
// weight traffic per product.  A 3x3 stride-1 conv uses 8 x 16-pixel tiles and loads,
// per 16-channel block, one halo box (16 x (16 sub + 2) pixels from column ow0 - 1)
// and the block's weights for all nine taps: each tap is the same box seen through a
// shifted operand descriptor (start ((row + kh) * 16 + kw) * 32 bytes, 8-row groups
// 512 bytes apart), so the input is copied about 1.8 times instead of nine:
//  * warp 0, lane 0: TMA producer.  Per K step one box of the input — 16 channels
//    x (wt x ht pixels, element stride = the conv stride) x 4 channel blocks,
//    started at the tap's offset (the zero padding comes from the out-of-bounds
//    fill) — and one box of the reference's packed weights [c1][k*k][co64][16]
//    (16 channels x up to 256 output channels x 4 channel blocks), both with the
//    32-byte swizzle: every 16-channel row is one K=16 slice of a K-major UMMA
//    operand (8-row groups 256 bytes apart).  A ring of as many stages as fit
//    in shared memory (up to 8), with full/empty mbarriers.
//  * warp 1, lane 0: MMA issuer into one of two TMEM accumulators (2 x 256
//    columns), committing each stage back to its empty barrier and each finished
//    tile to the accumulator's full barrier.
//  * warps 2-17: epilogue.  Warp w reads TMEM lanes 32(w%4).. (its 32 pixels) and
//    every fourth 16-column chunk, adds the bias, applies the SiLU, rounds once and
//    stores 32-byte NC1HWC0 rows (or NCHW elements); then frees the accumulator,
//    so tile t's stores overlap tile t+1's products.  Sixteen warps (four per lane
//    quarter) keep enough work in flight to hide the latency of the SiLU chain.
// Every wait is bounded (200 ms of wall time); a role that gives up records the
// reason in a device word (ttn_conv2d_fault_f16: 1 = copy, 2 = stage, 4 =
// accumulator), stops, and the CTA drains its copies and frees its TMEM.
#include <atomic>

#include "tcgen05.cuh"

namespace ttn {
namespace {

using namespace tc;

constexpr int kConvM = 128;          // output pixels per tile (UMMA M, TMEM lanes)
constexpr int kConvMaxN = 256;       // output channels per tile (UMMA N, TMEM columns per accumulator)
constexpr int kConvMaxStages = 8;    // shared-memory ring depth: as many stages as fit, up to 8
constexpr int kConvBlocksPerStep = 4;  // 16-channel blocks (K=16 each) per ring stage
constexpr int kConvEpiWarps = 16;
constexpr int kHaloW = 16;  // halo box width (pixels) for 8-pixel-wide 3x3 tiles: 512-byte rows keep
                            // every 8-row operand group on a 256-byte swizzle atom
constexpr int kConvThreads = 64 + 32 * kConvEpiWarps;

__device__ uint32_t g_conv_fault;

// Test hook (ttn_conv2d_test_withhold_copies): the next convolution launch issues
// no input copy.
std::atomic<bool> g_withhold_next_conv{false};

struct ConvArgs {
  const uint16_t* bias;  // fp16 [co] or null
  const uint16_t* res;   // NC1HWC0 residual of the output's shape, or null
  uint16_t* out;
  int64_t out_bs;        // elements between images of the output
  int64_t res_bs;        // elements between images of the residual
  int c1, oh, ow, co, kernel, stride, pad;
  int wt, ht;            // output sub-tile: wt x ht pixels, wt * ht = 128
  int tile_w, tile_h;    // output pixels per tile along w and h (both sub-tiles)
  int sub_dw, sub_dh;    // offset of sub-tile 1 from sub-tile 0 (0 and ht, or wt and 0)
  int tiles_w, tiles_h, co_tiles, tile_n;
  int blocks;            // channel blocks per step: min(4, c1)
  int groups;            // steps per tap: ceil(c1 / blocks)
  int64_t tiles;         // batch * tiles_h * tiles_w * co_tiles
  int silu, nchw;
  int bias_vec;          // the bias is 32-byte aligned: 16 channels in one 32-byte load
  int row32;             // output (and residual) rows are 32-byte aligned: one 32-byte access per pixel row
  int stages;           // ring depth
  int sub;               // pixel sub-tiles per tile (2 when tile_n <= 128: they share each weight stage)
  int halo;              // 3x3 stride 1: one halo box per channel block, the taps as shifted descriptors
  int steps;             // ring stages per tile
  int withhold;          // test hook: the producer issues no copy, so every other role's first wait runs out
  uint32_t a_box, a_bytes, b_off, b_bytes, stage_bytes;  // shared-memory layout of one stage
};
struct ConvMaps {
  CUtensorMap x, w;
};

// 32-byte global accesses (one 256-bit load or store per lane); the address must be
// 32-byte aligned.
__device__ __forceinline__ void ld_global_v8(const uint16_t* p, uint32_t (&w)[8]) {
  asm volatile("ld.global.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
               : "l"(p));
}
__device__ __forceinline__ void st_global_v8(uint16_t* p, const uint32_t (&w)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]),
               "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// Bias and activation of N accumulator columns (output channels co0 .. co0 + N - 1 of
// one pixel), packed in fp16 pairs: fp16(silu_f32(acc + bias)) or fp16(acc + bias), the
// bias added in FP32 where the channel exists: from `bias_words` (the N values, loaded by
// the caller ahead of the tensor-memory load) when `bias_vec`, else element by element.
// The SiLU is silu_pair_fast;
// lanes it flags take silu_f32 itself, so each output is exactly fp16(silu_f32(s)).
// fp16(x sigmoid(x)) for two FP32 values from silu_pair_fast's ex2/rcp core, rounded
// once without its bracket: within ~2^-19 (relative) of silu_f32, so an output can be
// the neighbouring fp16 value where silu_f32's result sits that close to a rounding
// midpoint.  `big` is set where a0 a1 >= 2^126 (a NaN, -inf, or inputs so negative
// that the shared reciprocal underflows): those lanes take silu_f32.
__device__ __forceinline__ uint32_t silu_pair_plain(unsigned long long xx, bool& big) {
  const unsigned long long t = f2_mul(xx, f2_pack(-1.44269504088896341f, -1.44269504088896341f));
  const float2 tt = f2_unpack(t);
  const float2 aa = f2_unpack(f2_add(f2_pack(ex2_approx(tt.x), ex2_approx(tt.y)), f2_pack(1.0f, 1.0f)));
  const float p = aa.x * aa.y, q = rcp_approx(p);
  const float2 r = f2_unpack(f2_mul(xx, f2_mul(f2_pack(aa.y, aa.x), f2_pack(q, q))));
  big = !(p < 8.50705917302346159e+37f);  // 2^126
  return h2_bits(__floats2half2_rn(r.x, r.y));
}

template <int N, bool kBracket = true>
__device__ __forceinline__ void conv_epilogue(const uint32_t (&r)[N], bool bias_vec, const uint32_t (&bias_words)[N / 2],
                                              const uint16_t* bias, int co0, int co, bool silu,
                                              uint32_t (&packed)[N / 2]) {
  constexpr int P = N / 2;
  unsigned long long v[P];
#pragma unroll
  for (int e = 0; e < P; ++e) v[e] = f2_pack(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
  if (bias) {
    if (bias_vec) {  // bias_words: the N fp16 bias values, loaded by the caller
#pragma unroll
      for (int e = 0; e < P; ++e) {
        const float2 b = __half22float2(bits_h2(bias_words[e]));
        v[e] = f2_add(v[e], f2_pack(b.x, b.y));
      }
    } else {
#pragma unroll
      for (int e = 0; e < P; ++e) {
        float2 s = f2_unpack(v[e]);
        if (co0 + 2 * e < co) s.x = __fadd_rn(s.x, __half2float(__ushort_as_half(bias[co0 + 2 * e])));
        if (co0 + 2 * e + 1 < co) s.y = __fadd_rn(s.y, __half2float(__ushort_as_half(bias[co0 + 2 * e + 1])));
        v[e] = f2_pack(s.x, s.y);
      }
    }
  }
  if (silu && !kBracket) {
    bool big[P], any = false;
#pragma unroll
    for (int e = 0; e < P; ++e) {
      packed[e] = silu_pair_plain(v[e], big[e]);
      any |= big[e];
    }
    if (any) {
#pragma unroll
      for (int e = 0; e < P; ++e)
        if (big[e]) {
          const float2 s = f2_unpack(v[e]);
          packed[e] = h2_bits(__floats2half2_rn(silu_f32(s.x), silu_f32(s.y)));
        }
    }
  } else if (silu) {
    uint32_t lower[P], open = 0;
#pragma unroll
    for (int e = 0; e < P; ++e) {
      packed[e] = silu_pair_fast(v[e], lower[e]);
      open |= packed[e] ^ lower[e];
    }
    if (open) {
#pragma unroll
      for (int e = 0; e < P; ++e) {
        const uint32_t diff = packed[e] ^ lower[e];
        if (diff) {
          const float2 s = f2_unpack(v[e]);
          if (diff & 0xffffu) packed[e] = (packed[e] & 0xffff0000u) | hbits(__float2half_rn(silu_f32(s.x)));
          if (diff >> 16) packed[e] = (packed[e] & 0x0000ffffu) | ((uint32_t)hbits(__float2half_rn(silu_f32(s.y))) << 16);
        }
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < P; ++e) {
      const float2 s = f2_unpack(v[e]);
      packed[e] = h2_bits(__floats2half2_rn(s.x, s.y));
    }
  }
}


template <bool kResidual>
__global__ void __launch_bounds__(kConvThreads, 1) conv_tc(ConvArgs a, const __grid_constant__ ConvMaps maps) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ __align__(8) uint64_t bars[2 * kConvMaxStages + 4];  // full[s], empty[s], acc_full[2], acc_empty[2]
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t a_box = a.a_box, a_bytes = a.a_bytes, b_off = a.b_off, b_bytes = a.b_bytes;
  const uint32_t stage_bytes = a.stage_bytes;
  const uint32_t smem0 = ((uint32_t)__cvta_generic_to_shared(smem) + 1023u) & ~1023u;
  const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(&bars[0]);
  auto full_bar = [&](int s) { return bar0 + 8 * s; };
  const int stages = a.stages;
  auto empty_bar = [&](int s) { return bar0 + 8 * (kConvMaxStages + s); };
  auto acc_full = [&](int i) { return bar0 + 8 * (2 * kConvMaxStages + i); };
  auto acc_empty = [&](int i) { return bar0 + 8 * (2 * kConvMaxStages + 2 + i); };
  const int64_t stride = gridDim.x;
  const int count = a.tiles > (int64_t)blockIdx.x ? (int)((a.tiles - blockIdx.x + stride - 1) / stride) : 0;
  const int steps = a.steps;
  // tile j of this CTA -> image, output-pixel origin, first output channel
  auto tile_coords = [&](int j, int& img, int& oh0, int& ow0, int& n0) {  // 32-bit: tiles < 2^31
    uint32_t t = blockIdx.x + (uint32_t)j * gridDim.x;
    n0 = (int)(t % (uint32_t)a.co_tiles) * a.tile_n;
    t /= (uint32_t)a.co_tiles;
    ow0 = (int)(t % (uint32_t)a.tiles_w) * a.tile_w;
    t /= (uint32_t)a.tiles_w;
    oh0 = (int)(t % (uint32_t)a.tiles_h) * a.tile_h;
    img = (int)(t / (uint32_t)a.tiles_h);
  };

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(acc_full(i), 1);
      mbar_init(acc_empty(i), kConvEpiWarps);
    }
    mbar_init_fence();
  }
  if (warp == 1) tmem_alloc((uint32_t)__cvta_generic_to_shared(&tmem_slot), 2 * kConvMaxN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  uint32_t fault = 0;

  if (warp == 0 && lane == 0) {  // TMA producer
    uint32_t fills[kConvMaxStages] = {0, 0, 0, 0, 0, 0, 0, 0};
    int s = 0;
    uint32_t phase = 0;
    bool ok = !a.withhold;
    for (int j = 0; j < count && ok; ++j) {
      int img, oh0, ow0, n0;
      tile_coords(j, img, oh0, ow0, n0);
      for (int step = 0; step < steps; ++step) {
        if (!mbar_wait(empty_bar(s), phase ^ 1)) {  // a fresh barrier counts as freed
          fault |= 2u;
          ok = false;
          break;
        }
        const uint32_t sa = smem0 + s * stage_bytes, sb = sa + b_off;
        mbar_expect_tx(full_bar(s), a_bytes + b_bytes);
        if (a.halo) {  // step = channel block: its 16 x (sub*ht+2) halo and its weights of all 9 taps
          tma_load5(sa, &maps.x, 0, ow0 - 1, oh0 - 1, step, img, full_bar(s));
          tma_load4(sb, &maps.w, 0, n0, 0, step, full_bar(s));
        } else {
          const int tap = step / a.groups, cb = (step % a.groups) * a.blocks;
          const int kh = tap / a.kernel, kw = tap % a.kernel;
          for (int u = 0; u < a.sub; ++u)
            tma_load5(sa + u * a_box, &maps.x, 0, (ow0 + u * a.sub_dw) * a.stride + kw - a.pad,
                      (oh0 + u * a.sub_dh) * a.stride + kh - a.pad, cb, img, full_bar(s));
          tma_load4(sb, &maps.w, 0, n0, tap, cb, full_bar(s));
        }
        ++fills[s];
        if (++s == stages) s = 0, phase ^= 1;
      }
    }
    for (int i = 0; i < stages; ++i)  // copies in flight after an early exit (bounded)
      if (fills[i] && !mbar_wait(full_bar(i), (fills[i] - 1) & 1)) fault |= 1u;
  } else if (warp == 1 && lane == 0) {  // MMA issuer
    const uint32_t idesc = umma_idesc(kConvM, a.tile_n, false, false);
    int s = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int j = 0; j < count && ok; ++j) {
      const int acc = j & 1;
      if (!mbar_wait(acc_empty(acc), ((j >> 1) & 1) ^ 1)) {
        fault |= 4u;
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem + acc * kConvMaxN;  // sub-tile u at d + u * tile_n (sub = 2: tile_n <= 128)
      for (int step = 0; step < steps; ++step) {
        if (!mbar_wait(full_bar(s), phase)) {
          fault |= 1u;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem0 + s * stage_bytes, sb = sa + b_off;
        // Descriptors are built once per stage and stepped by adding (byte offset >> 4) to the start
        // field (shared-memory addresses stay below 256 KB: no carry); one thread issues every
        // product, so its per-product instruction count sets the issue rate.
        const bool acc0 = step > 0;
        if (a.halo) {  // tap (kh, kw) of sub-tile u: the halo shifted by (u*ht + kh) rows and kw pixels;
                       // 8-pixel tile rows are the operand's 8-row groups, kHaloW*32 bytes apart
          const uint64_t a0 = smem_desc(sa, 16, kHaloW * 32, kSwizzle32B), b0 = smem_desc(sb, 16, 256, kSwizzle32B);
          const uint32_t sub_off = (uint32_t)(a.ht * kHaloW * 32) >> 4, bn = (uint32_t)(a.tile_n * 32) >> 4;
#pragma unroll
          for (int tap = 0; tap < 9; ++tap) {
            const uint64_t ad = a0 + ((tap / 3) * kHaloW * 2 + (tap % 3) * 2), bd = b0 + tap * bn;
            const bool acc = acc0 || tap > 0;
            umma_ss(d, ad, bd, idesc, acc);
            if (a.sub == 2) umma_ss(d + a.tile_n, ad + sub_off, bd, idesc, acc);
          }
        } else {
          const uint64_t a0 = smem_desc(sa, 16, 256, kSwizzle32B), b0 = smem_desc(sb, 16, 256, kSwizzle32B);
          const uint32_t bi = (uint32_t)(a.tile_n * 32) >> 4, ab = a_box >> 4;
#pragma unroll
          for (int i = 0; i < kConvBlocksPerStep; ++i)
            if (i < a.blocks) {
              const uint64_t ad = a0 + i * (kConvM * 32 / 16), bd = b0 + i * bi;
              const bool acc = acc0 || i > 0;
              umma_ss(d, ad, bd, idesc, acc);
              if (a.sub == 2) umma_ss(d + a.tile_n, ad + ab, bd, idesc, acc);
            }
        }
        umma_commit(empty_bar(s));  // the stage is free once these products have read it
        if (++s == stages) s = 0, phase ^= 1;
      }
      if (ok) umma_commit(acc_full(acc));
    }
  } else if (warp >= 2) {  // epilogue
    // Warp w reads TMEM lanes 32 (w % 4) .. (its 32 pixels of each sub-tile) and every
    // fourth 16-column chunk of the accumulator, starting at chunk (w - 2) / 4.  The
    // chunk count, sub * tile_n / 16, is 4, 8, 12 or 16: the four warps of a lane
    // quarter take the same number.
    constexpr int kGroups = kConvEpiWarps / 4;
    const int quarter = warp & 3, group = (warp - 2) >> 2, m = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const int th = m / a.wt, tw = m % a.wt;
    const int chunks = a.sub * a.tile_n / 16;
    for (int j = 0; j < count; ++j) {
      const int acc = j & 1;
      if (!mbar_wait(acc_full(acc), (j >> 1) & 1)) {
        fault |= 4u;
        break;
      }
      tc_fence_after();
      int img, oh0, ow0, n0;
      tile_coords(j, img, oh0, ow0, n0);
      uint16_t* out = a.out + img * a.out_bs;
      for (int c = group; c < chunks; c += kGroups) {
        const int u = c * 16 >= a.tile_n ? 1 : 0;  // sub-tile 1: sub_dh rows down or sub_dw pixels on
        const int co0 = n0 + c * 16 - u * a.tile_n, oh = oh0 + u * a.sub_dh + th, ow = ow0 + u * a.sub_dw + tw;
        // the chunk's bias first (one address for the whole warp), so its latency overlaps the
        // tensor-memory load's: the load's wait orders every later memory access behind it
        const bool bias_vec = a.bias && a.bias_vec && co0 + 16 <= a.co;
        uint32_t bias_words[8];
        if (bias_vec) ld_global_v8(a.bias + co0, bias_words);
        uint32_t r[16];
        __syncwarp();  // the tensor-memory load is warp-collective: reconverge after the stores
        tmem_ld16(lane_addr + acc * kConvMaxN + c * 16, r);
        if (oh >= a.oh || ow >= a.ow || co0 >= a.co) continue;
        uint32_t packed[8];
        conv_epilogue<16, false>(r, bias_vec, bias_words, a.bias, co0, a.co, a.silu, packed);
        if (a.nchw) {
          const int64_t plane = (int64_t)a.oh * a.ow;
          uint16_t* o = out + (int64_t)co0 * plane + (int64_t)oh * a.ow + ow;
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (co0 + e < a.co) o[e * plane] = (uint16_t)(packed[e / 2] >> (16 * (e & 1)));
        } else {  // co is a multiple of 16: the chunk is one whole 16-channel block
          const int64_t at = (((int64_t)(co0 / 16) * a.oh + oh) * a.ow + ow) << 4;
          if (kResidual) {  // the reference's separate fp16 add: fp16(float(res) + float(y))
            const uint16_t* rp = a.res + img * a.res_bs + at;
            uint32_t rv[8];
            if (a.row32) {
              ld_global_v8(rp, rv);
            } else {
              const uint4 q0 = reinterpret_cast<const uint4*>(rp)[0], q1 = reinterpret_cast<const uint4*>(rp)[1];
              rv[0] = q0.x, rv[1] = q0.y, rv[2] = q0.z, rv[3] = q0.w, rv[4] = q1.x, rv[5] = q1.y, rv[6] = q1.z,
              rv[7] = q1.w;
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float2 y2 = __half22float2(bits_h2(packed[e]));
              const float2 r2 = __half22float2(bits_h2(rv[e]));
              packed[e] = h2_bits(__floats2half2_rn(__fadd_rn(r2.x, y2.x), __fadd_rn(r2.y, y2.y)));
            }
          }
          if (a.row32) {
            st_global_v8(out + at, packed);  // the pixel's whole 32-byte row: full sectors
          } else {
            uint4* o = reinterpret_cast<uint4*>(out + at);
            o[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            o[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty(acc));
    }
  }
  if (fault) atomicOr(&g_conv_fault, fault);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kConvMaxN);
  }
}

// packed[cb][tap][co64][16] = w[co][cb * 16 + c][tap], zero where co >= co or ci >= ci
// (the reference's prepare(): conv_img.cpp:321-383, blocked_c2f.py:66).
__global__ void conv_pack_weights(const uint16_t* __restrict__ w, uint16_t* __restrict__ packed, int co, int ci,
                                  int taps, int co_pad, int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % 16);
    int64_t t = i / 16;
    const int o = (int)(t % co_pad);
    t /= co_pad;
    const int tap = (int)(t % taps);
    const int cb = (int)(t / taps);
    const int cin = cb * 16 + c;
    packed[i] = (o < co && cin < ci) ? w[((int64_t)o * ci + cin) * taps + tap] : (uint16_t)0;
  }
}

int gcd_int(int x, int y) {
  while (y) {
    const int t = x % y;
    x = y;
    y = t;
  }
  return x;
}

// The stem convolution -- one input channel block, 3x3, stride 2 (YOLO's first
// layer: 3 real channels padded to 16).  Weights that use at most three input
// channels go to conv_stem_tc (below: a 27-long reduction on the tensor cores);
// wider ones run here on the CUDA cores (conv_tc would re-read every tap through
// 32-byte TMA rows).  Each output pixel reads its nine input rows once (neighbours
// share them in L1) and only the input channels the weights use: the block finds
// the highest channel with a nonzero
// weight (input channels past the real count are zero by contract) and takes the
// body compiled for that many channels (1-4, 8 or 16), so the channel loops are
// static.  Thread = PIX adjacent output pixels x the 16 output channels of its
// block's channel group (grid y); the group's weights sit in shared memory as FP32
// pairs of output channels, so each (channel, tap) is one broadcast load and one
// f32x2 FMA per pixel and channel pair.  Epilogue: +
// bias, then fp16(silu_f32) as the tensor-core kernel rounds it, from the bracketed
// ex2/rcp core (silu_pair_fast) with silu_f32 itself for the lanes it flags; NC1HWC0
// output, 32 bytes per channel block.
constexpr int kStemThreads = 128;

struct StemArgs {
  const uint16_t* x;
  int64_t x_bs;
  int h, w, oh, ow, batch, silu;
  uint16_t* out;
  int64_t out_bs;
};

template <int CO, int PIX, int CE>
__device__ void stem_pixels(const StemArgs& a, const unsigned long long* wsm, const float* bsm) {
  constexpr int PAIRS = CO / 2;  // CO: the output channels of this block's group
  const int groups_w = (a.ow + PIX - 1) / PIX;
  const int64_t total = (int64_t)a.batch * a.oh * groups_w;
  for (int64_t t = (int64_t)blockIdx.x * kStemThreads + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * kStemThreads) {
    const int64_t b = t / ((int64_t)a.oh * groups_w);
    const int r = (int)(t - b * a.oh * groups_w), oy = r / groups_w, ox0 = (r - oy * groups_w) * PIX;
    const uint16_t* img = a.x + b * a.x_bs;
    unsigned long long acc[PIX][PAIRS];
#pragma unroll
    for (int p = 0; p < PIX; ++p)
#pragma unroll
      for (int q = 0; q < PAIRS; ++q) acc[p][q] = 0ull;
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
      const int iy = 2 * oy - 1 + tap / 3;
      uint32_t words[PIX][(CE + 1) / 2];  // the used channels' fp16 pairs
#pragma unroll
      for (int p = 0; p < PIX; ++p) {
        const int ix = 2 * (ox0 + p) - 1 + tap % 3;
        const bool in = iy >= 0 && iy < a.h && ix >= 0 && ix < a.w && ox0 + p < a.ow;
        const uint16_t* src = img + ((int64_t)iy * a.w + ix) * 16;
        if constexpr (CE <= 4) {
          const uint2 v = in ? __ldg(reinterpret_cast<const uint2*>(src)) : make_uint2(0u, 0u);
          words[p][0] = v.x;
          if constexpr (CE > 2) words[p][1] = v.y;
        } else {
#pragma unroll
          for (int hv = 0; hv < CE / 8; ++hv) {
            const uint4 v = in ? __ldg(reinterpret_cast<const uint4*>(src) + hv) : make_uint4(0u, 0u, 0u, 0u);
            words[p][4 * hv] = v.x, words[p][4 * hv + 1] = v.y, words[p][4 * hv + 2] = v.z, words[p][4 * hv + 3] = v.w;
          }
        }
      }
#pragma unroll
      for (int c = 0; c < CE; ++c) {
        const unsigned long long* wc = wsm + (c * 9 + tap) * PAIRS;
        unsigned long long xv[PIX];
#pragma unroll
        for (int p = 0; p < PIX; ++p) {
          const float v = __half2float(__ushort_as_half((uint16_t)(words[p][c >> 1] >> (16 * (c & 1)))));
          xv[p] = f2_pack(v, v);
        }
#pragma unroll
        for (int q = 0; q < PAIRS; ++q) {
          const unsigned long long wq = wc[q];
#pragma unroll
          for (int p = 0; p < PIX; ++p) acc[p][q] = f2_fma(xv[p], wq, acc[p][q]);
        }
      }
    }
    uint16_t* dst = a.out + b * a.out_bs + (int64_t)blockIdx.y * a.oh * a.ow * 16;
#pragma unroll
    for (int p = 0; p < PIX; ++p) {
      if (ox0 + p >= a.ow) continue;
#pragma unroll
      for (int blk = 0; blk < CO / 16; ++blk) {
        uint32_t o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const unsigned long long sum =
              f2_add(acc[p][blk * 8 + e], f2_pack(bsm[blk * 16 + 2 * e], bsm[blk * 16 + 2 * e + 1]));
          if (!a.silu) {
            const float2 v = f2_unpack(sum);
            o[e] = h2_bits(__floats2half2_rn(v.x, v.y));
            continue;
          }
          uint32_t lower;
          o[e] = silu_pair_fast(sum, lower);  // fp16(silu_f32) unless flagged
          const uint32_t open = o[e] ^ lower;
          if (open) {
            const float2 v = f2_unpack(sum);
            if (open & 0xffffu) o[e] = (o[e] & 0xffff0000u) | __half_as_ushort(__float2half_rn(silu_f32(v.x)));
            if (open >> 16) o[e] = (o[e] & 0xffffu) | ((uint32_t)__half_as_ushort(__float2half_rn(silu_f32(v.y))) << 16);
          }
        }
        uint4* q = reinterpret_cast<uint4*>(dst + (((int64_t)blk * a.oh + oy) * a.ow + ox0 + p) * 16);
        q[0] = make_uint4(o[0], o[1], o[2], o[3]);
        q[1] = make_uint4(o[4], o[5], o[6], o[7]);
      }
    }
  }
}

// True (block-wide; every thread must call it) when any of the co output channels
// has a nonzero weight on an input channel past the third: the stem then needs the
// CUDA-core kernel, otherwise the tensor-core one (K = 27) takes it.  Both kernels
// decide from this same predicate, so exactly one of them does the work.
// Each (tap, output channel) weight row is 32 bytes (16 input channels), read as two
// 16-byte loads; a value is nonzero exactly when its bits without the sign are.
__device__ __forceinline__ bool stem_wide(const uint16_t* packed, int co64, int co) {
  uint32_t mine = 0;
  for (int i = threadIdx.x; i < 9 * co; i += blockDim.x) {
    const int tap = i / co, n = i - tap * co;
    const uint4* row = reinterpret_cast<const uint4*>(packed + ((int64_t)tap * co64 + n) * 16);
    const uint4 q0 = __ldg(row), q1 = __ldg(row + 1);
    mine |= (q0.y & 0x7fff0000u) | ((q0.z | q0.w | q1.x | q1.y | q1.z | q1.w) & 0x7fff7fffu);  // channels 3-15
  }
  return __syncthreads_or(mine != 0) != 0;
}

template <int CO, int PIX>
__global__ void __launch_bounds__(kStemThreads) conv_stem(StemArgs a, const uint16_t* packed, int co64,
                                                          const uint16_t* bias) {
  constexpr int PAIRS = CO / 2;
  const int group = blockIdx.y * CO;  // this block's first output channel
  __shared__ unsigned long long wsm[16 * 9 * PAIRS];  // [channel][tap][output pair] packed f32x2
  __shared__ float bsm[CO];
  __shared__ int used;
  const int tid = threadIdx.x;
  if (!stem_wide(packed, co64, (int)gridDim.y * CO)) return;  // conv_stem_tc takes it
  if (tid == 0) used = 0;
  __syncthreads();
  int mine = 0;
  for (int i = tid; i < 16 * 9 * PAIRS; i += kStemThreads) {
    const int q = i % PAIRS, rest = i / PAIRS, tap = rest % 9, c = rest / 9;
    const float w0 = __half2float(__ushort_as_half(packed[((int64_t)tap * co64 + group + 2 * q) * 16 + c]));
    const float w1 = __half2float(__ushort_as_half(packed[((int64_t)tap * co64 + group + 2 * q + 1) * 16 + c]));
    wsm[i] = f2_pack(w0, w1);
    if (w0 != 0.0f || w1 != 0.0f) mine = c + 1;
  }
  if (mine) atomicMax(&used, mine);
  for (int i = tid; i < CO; i += kStemThreads) bsm[i] = bias ? __half2float(__ushort_as_half(bias[group + i])) : 0.0f;
  __syncthreads();
  switch (used) {  // block-uniform
    case 0:
    case 1: stem_pixels<CO, PIX, 1>(a, wsm, bsm); break;
    case 2: stem_pixels<CO, PIX, 2>(a, wsm, bsm); break;
    case 3: stem_pixels<CO, PIX, 3>(a, wsm, bsm); break;
    case 4: stem_pixels<CO, PIX, 4>(a, wsm, bsm); break;
    case 5: case 6: case 7: case 8: stem_pixels<CO, PIX, 8>(a, wsm, bsm); break;
    default: stem_pixels<CO, PIX, 16>(a, wsm, bsm); break;
  }
}

// The stem on the tensor cores when its weights use input channels 0-2 only (the
// YOLO image): the reduction is 27 long (k = tap * 3 + channel, zero-padded to 32)
// instead of nine 16-channel taps.  A tile is 128 consecutive output pixels of one
// image.  Each thread gathers its pixel's 27 inputs (nine 8-byte loads, zeros past
// the border) into a 128 x 32 K-major operand in shared memory (two 32-byte rows per
// pixel, the 32-byte swizzle the descriptors name); the weights are a 32 x co operand
// built once per CTA.  One thread issues the two K = 16 products (M = 128, N = co)
// into tensor memory and commits them to an mbarrier; each warp then reads its 32
// pixels' accumulators in 16-column chunks and runs conv_tc's epilogue (bias,
// bracketed SiLU, one rounding, 32-byte NC1HWC0 rows).  Persistent CTAs, several per
// SM, so one CTA's gather overlaps another's epilogue.  The wait on the products is
// bounded; a CTA whose wait runs out sets bit 4 of the fault word and stops.
constexpr int kStemTcThreads = 128;
constexpr int kStemTcBlocks = 6;  // CTAs per SM (85 registers; TMEM 6 x 64 columns at most)

__global__ void __launch_bounds__(kStemTcThreads, kStemTcBlocks) conv_stem_tc(StemArgs a, const uint16_t* packed, int co64,
                                                                  int co, const uint16_t* bias, int bias_vec,
                                                                  int row32) {
  __shared__ __align__(1024) unsigned char a_tile[2 * kConvM * 32];  // [K block][pixel][32 bytes]
  __shared__ __align__(1024) unsigned char b_tile[2 * 64 * 32];      // [K block][output channel][32 bytes]
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, warp = tid >> 5;
  if (stem_wide(packed, co64, co)) return;  // conv_stem takes it
  const uint32_t sa = (uint32_t)__cvta_generic_to_shared(a_tile), sb = (uint32_t)__cvta_generic_to_shared(b_tile);
  const uint32_t bar_addr = (uint32_t)__cvta_generic_to_shared(&bar);
  const uint32_t cols = co <= 32 ? 32 : 64;
  // row r of a K-major operand, 16-byte half h: the 32-byte swizzle moves the half of rows 4-7
  // of every 8-row group
  auto swz = [](int r, int h) { return (uint32_t)(r * 32 + ((h ^ ((r >> 2) & 1)) << 4)); };
  for (int i = tid; i < co * 32; i += kStemTcThreads) {  // weights: row n, k = tap * 3 + channel
    const int n = i >> 5, k = i & 31, kb = k >> 4, kk = k & 15;
    const uint16_t v = k < 27 ? packed[((int64_t)(k / 3) * co64 + n) * 16 + k % 3] : (uint16_t)0;
    *reinterpret_cast<uint16_t*>(b_tile + kb * co * 32 + swz(n, kk >> 3) + (kk & 7) * 2) = v;
  }
  if (tid == 0) {
    mbar_init(bar_addr, 1);
    mbar_init_fence();
  }
  if (warp == 0) tmem_alloc((uint32_t)__cvta_generic_to_shared(&tmem_slot), cols);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot, lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
  const uint32_t idesc = umma_idesc(kConvM, co, false, false);
  const uint64_t adesc = smem_desc(sa, 16, 256, kSwizzle32B), bdesc = smem_desc(sb, 16, 256, kSwizzle32B);
  const int plane = a.oh * a.ow, tiles_img = (plane + kConvM - 1) / kConvM;
  const int64_t total = (int64_t)a.batch * tiles_img;
  uint32_t phase = 0;
  for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    const int64_t img = t / tiles_img;
    const int p = (int)(t - img * tiles_img) * kConvM + tid;
    const bool valid = p < plane;
    const int oy = valid ? p / a.ow : 0, ox = valid ? p - oy * a.ow : 0;
    {  // gather: this pixel's 27 inputs as one 64-byte K row (two swizzled 32-byte rows)
      const uint16_t* src = a.x + img * a.x_bs;
      uint16_t hv[32];
#pragma unroll
      for (int tap = 0; tap < 9; ++tap) {
        const int iy = 2 * oy - 1 + tap / 3, ix = 2 * ox - 1 + tap % 3;
        const bool in = valid && iy >= 0 && iy < a.h && ix >= 0 && ix < a.w;
        const uint2 v = in ? __ldg(reinterpret_cast<const uint2*>(src + ((int64_t)iy * a.w + ix) * 16))
                           : make_uint2(0u, 0u);
        hv[3 * tap] = (uint16_t)v.x, hv[3 * tap + 1] = (uint16_t)(v.x >> 16), hv[3 * tap + 2] = (uint16_t)v.y;
      }
#pragma unroll
      for (int k = 27; k < 32; ++k) hv[k] = 0;
#pragma unroll
      for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int k0 = kb * 16 + h * 8;
          uint4 q;
          q.x = hv[k0] | ((uint32_t)hv[k0 + 1] << 16), q.y = hv[k0 + 2] | ((uint32_t)hv[k0 + 3] << 16);
          q.z = hv[k0 + 4] | ((uint32_t)hv[k0 + 5] << 16), q.w = hv[k0 + 6] | ((uint32_t)hv[k0 + 7] << 16);
          *reinterpret_cast<uint4*>(a_tile + kb * kConvM * 32 + swz(tid, h)) = q;
        }
    }
    fence_proxy_async_smem();  // the generic stores above, before the products read them
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      umma_ss(tmem, adesc, bdesc, idesc, false);
      umma_ss(tmem, adesc + ((kConvM * 32) >> 4), bdesc + ((uint32_t)(co * 32) >> 4), idesc, true);
      umma_commit(bar_addr);
    }
    if (!__syncthreads_and(mbar_wait(bar_addr, phase))) {
      atomicOr(&g_conv_fault, 4u);
      break;
    }
    phase ^= 1;
    tc_fence_after();
    uint16_t* out = a.out + img * a.out_bs;
    for (int c0 = 0; c0 < co; c0 += 16) {
      const bool bv = bias && bias_vec;
      uint32_t bias_words[8];
      if (bv) ld_global_v8(bias + c0, bias_words);
      uint32_t r[16];
      __syncwarp();
      tmem_ld16(lane_addr + c0, r);
      if (!valid) continue;
      uint32_t packed_out[8];
      conv_epilogue<16, false>(r, bv, bias_words, bias, c0, co, a.silu, packed_out);
      uint16_t* o = out + (((int64_t)(c0 / 16) * a.oh + oy) * a.ow + ox) * 16;
      if (row32) {
        st_global_v8(o, packed_out);
      } else {
        reinterpret_cast<uint4*>(o)[0] = make_uint4(packed_out[0], packed_out[1], packed_out[2], packed_out[3]);
        reinterpret_cast<uint4*>(o)[1] = make_uint4(packed_out[4], packed_out[5], packed_out[6], packed_out[7]);
      }
    }
    tc_fence_before();
    __syncthreads();  // the accumulators and the operand tile are free for the next tile
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, cols);
  }
}

}  // namespace
}  // namespace ttn

using namespace ttn;

namespace {

ttn_status conv_launch(const char* name, const void* x, int64_t batch, int64_t c1, int64_t h, int64_t w,
                       int64_t x_batch_stride, const void* packed_weights, const void* bias, int64_t co,
                       int32_t kernel, int32_t stride, uint32_t flags, const void* residual,
                       int64_t residual_batch_stride, void* out, int64_t out_batch_stride, ttn_stream stream) {
  if (flags & ~(TTN_CONV_SILU | TTN_CONV_NCHW)) return fail(TTN_INVALID_ARG, "%s: unknown flags %u", name, flags);
  if (batch < 0 || c1 <= 0 || h <= 0 || w <= 0 || co <= 0)
    return fail(TTN_INVALID_ARG, "%s: sizes must be positive (batch >= 0)", name);
  if (!((kernel == 1 && stride == 1) || ((kernel == 3 || kernel == 6) && (stride == 1 || stride == 2))))
    return fail(TTN_UNSUPPORTED, "%s: 1x1 stride 1, or 3x3 / 6x6 stride 1 or 2", name);
  const bool nchw = flags & TTN_CONV_NCHW;
  if (!nchw && co % 16) return fail(TTN_UNSUPPORTED, "%s: NC1HWC0 output needs co % 16 == 0", name);
  const int pad = (kernel - 1) / 2;
  const int64_t oh = (h + 2 * pad - kernel) / stride + 1, ow = (w + 2 * pad - kernel) / stride + 1;
  if (oh <= 0 || ow <= 0) return fail(TTN_INVALID_ARG, "%s: kernel exceeds the padded input", name);
  if (!batch) return TTN_OK;
  if (!x || !packed_weights || !out) return fail(TTN_INVALID_ARG, "%s: null pointer", name);
  if (((uintptr_t)x | (uintptr_t)packed_weights | (uintptr_t)out) & 15u || x_batch_stride % 8 ||
      out_batch_stride % 8 || (bias && ((uintptr_t)bias & 1u)))
    return fail(TTN_INVALID_ARG, "%s: 16-byte aligned tensors and batch strides that are multiples of 8", name);
  const int64_t per_image = c1 * h * w * 16, out_image = (nchw ? co : co / 16 * 16) * oh * ow;
  if (x_batch_stride < per_image && batch > 1)
    return fail(TTN_INVALID_ARG, "%s: input images overlap", name);
  if (out_batch_stride < out_image && batch > 1)
    return fail(TTN_INVALID_ARG, "%s: output images overlap", name);
  if (c1 > 65535 || h > 65535 || w > 65535 || co > 65536 || batch > INT32_MAX)
    return fail(TTN_UNSUPPORTED, "%s: shape beyond the supported range", name);
  if (c1 == 1 && kernel == 3 && stride == 2 && !nchw && !residual && co <= 64) {  // the stem
    const dim3 grid(grid_for(batch * oh * ((ow + 1) / 2), kStemThreads, 16), (unsigned)(co / 16));
    const StemArgs a{(const uint16_t*)x, batch > 1 ? x_batch_stride : 0, (int)h, (int)w, (int)oh, (int)ow,
                     (int)batch, (flags & TTN_CONV_SILU) ? 1 : 0, (uint16_t*)out, batch > 1 ? out_batch_stride : 0};
    // both launch; from the weights each block decides whether its kernel applies (at most
    // three input channels used: the tensor cores; more: the CUDA cores)
    const int64_t tiles = batch * ((oh * ow + kConvM - 1) / kConvM);
    const int64_t slots = (int64_t)sm_count() * kStemTcBlocks;
    const unsigned grid_tc = (unsigned)(tiles < slots ? tiles : slots);
    const int bias_vec = bias && ((uintptr_t)bias & 31u) == 0 ? 1 : 0;
    const int row32 = ((uintptr_t)out & 31u) == 0 && (batch == 1 || out_batch_stride % 16 == 0) ? 1 : 0;
    conv_stem_tc<<<grid_tc, kStemTcThreads, 0, (cudaStream_t)stream>>>(
        a, (const uint16_t*)packed_weights, (int)((co + 63) / 64 * 64), (int)co, (const uint16_t*)bias, bias_vec,
        row32);
    TTN_TRY(launch_check(name));
    conv_stem<16, 2><<<grid, kStemThreads, 0, (cudaStream_t)stream>>>(a, (const uint16_t*)packed_weights,
                                                                       (int)((co + 63) / 64 * 64),
                                                                       (const uint16_t*)bias);
    return launch_check(name);
  }
  if (residual) {
    if (nchw) return fail(TTN_UNSUPPORTED, "%s: the residual needs NC1HWC0 output", name);
    if (((uintptr_t)residual & 15u) || residual_batch_stride % 8)
      return fail(TTN_INVALID_ARG, "%s: 16-byte aligned residual, batch stride a multiple of 8", name);
  }
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return fail(TTN_CUDA_ERROR, "%s: cuTensorMapEncodeTiled is not available", name);

  // A 1x1 conv (stride 1) has no spatial neighbourhood: each image is one row of h * w
  // pixels, so a tile is 128 consecutive pixels (its sub-tile the next 128) whatever the
  // image's shape, and pads at most the image's last tile.
  const bool flat = kernel == 1;
  if (flat && h * w > INT32_MAX) return fail(TTN_UNSUPPORTED, "%s: more than 2^31 pixels per image", name);
  const int64_t gh = flat ? 1 : h, gw = flat ? h * w : w, goh = flat ? 1 : oh, gow = flat ? oh * ow : ow;

  ConvArgs a;
  a.bias = (const uint16_t*)bias;
  a.res = (const uint16_t*)residual;
  a.out = (uint16_t*)out;
  a.out_bs = out_batch_stride;
  a.res_bs = batch > 1 ? residual_batch_stride : 0;
  a.c1 = (int)c1, a.oh = (int)goh, a.ow = (int)gow, a.co = (int)co;
  a.kernel = kernel, a.stride = stride, a.pad = pad;
  // every 3x3 stride-1 conv takes the 8-pixel-wide halo tiles, two sub-tiles (16 rows each) sharing
  // the weights where tile_n <= 128 even when that pads the last tile's rows (80 rows -> 96): on a B200
  // that beat the plain 16 x 16 tiles at 80x80 (128 -> 128: 118 -> 83 us), which reload the input per tap
  a.halo = kernel == 3 && stride == 1;
  a.wt = a.halo ? 8 : flat ? kConvM : gcd_int((int)ow, kConvM);  // halo: one 8-pixel row per 8-row operand group
  a.ht = kConvM / a.wt;
  const int64_t co_pad = (co + 63) / 64 * 64;
  a.tile_n = (int)(co_pad < kConvMaxN ? co_pad : kConvMaxN);
  {  // two sub-tiles (the next ht rows, or flat the next 128 pixels) share the weight stages when
     // they fit the accumulators and, except for halo tiles, pad no extra pixels
    const int64_t len = flat ? gow : goh, step = flat ? a.wt : a.ht;
    const int64_t pad1 = (len + step - 1) / step * step, pad2 = (len + 2 * step - 1) / (2 * step) * (2 * step);
    a.sub = a.tile_n <= kConvMaxN / 2 && (pad2 <= pad1 || a.halo) ? 2 : 1;
  }
  a.sub_dw = flat ? a.wt : 0;
  a.sub_dh = flat ? 0 : a.ht;
  auto geometry = [&]() {
    a.tile_w = flat ? a.sub * a.wt : a.wt;
    a.tile_h = flat ? a.ht : a.sub * a.ht;
    a.tiles_w = (int)((gow + a.tile_w - 1) / a.tile_w);
    a.tiles_h = (int)((goh + a.tile_h - 1) / a.tile_h);
    a.co_tiles = (int)((co_pad + a.tile_n - 1) / a.tile_n);
  };
  geometry();
  if (a.tile_n == kConvMaxN && a.sub == 1) {
    // Wave quantization: where the 256-channel tiles leave the last round of the persistent
    // CTAs mostly idle (a few hundred tiles on 148 SMs), 128-channel tiles (one sub-tile)
    // take at least 16% fewer tile-rounds of work for ~12% more operand bytes (on a B200:
    // 3x3 256 -> 256 at 20x20, batch 32, 64.6 -> 50.5 us; outputs bit-identical).
    const int64_t sms = sm_count(), per_co = batch * a.tiles_w * a.tiles_h;
    const int64_t rounds256 = (per_co * a.co_tiles + sms - 1) / sms;
    const int64_t rounds128 = (per_co * ((co_pad + 127) / 128) + sms - 1) / sms;
    if (rounds128 * 128 * 100 <= rounds256 * kConvMaxN * 84) {
      a.tile_n = kConvMaxN / 2;
      geometry();
    }
  }
  a.blocks = a.halo ? 1 : (int)(c1 < kConvBlocksPerStep ? c1 : kConvBlocksPerStep);
  a.groups = (int)((c1 + a.blocks - 1) / a.blocks);
  a.steps = a.halo ? (int)c1 : kernel * kernel * a.groups;
  if (a.halo) {
    a.a_box = a.a_bytes = (uint32_t)((a.sub * a.ht + 2) * kHaloW * 32);
    a.b_bytes = (uint32_t)(9 * a.tile_n * 32);
  } else {
    a.a_box = (uint32_t)(a.blocks * kConvM * 32);
    a.a_bytes = a.a_box * a.sub;
    a.b_bytes = (uint32_t)(a.blocks * a.tile_n * 32);
  }
  a.b_off = (a.a_bytes + 1023u) & ~1023u;
  a.stage_bytes = (a.b_off + a.b_bytes + 1023u) & ~1023u;
  a.tiles = batch * a.tiles_h * a.tiles_w * a.co_tiles;
  if (a.tiles >= ((int64_t)1 << 31)) return fail(TTN_UNSUPPORTED, "%s: more than 2^31 output tiles", name);
  a.silu = (flags & TTN_CONV_SILU) ? 1 : 0;
  a.nchw = nchw ? 1 : 0;
  a.bias_vec = bias && ((uintptr_t)bias & 31u) == 0 ? 1 : 0;
  a.row32 = ((uintptr_t)out & 31u) == 0 && (batch == 1 || out_batch_stride % 16 == 0) &&
            (!residual || (((uintptr_t)residual & 31u) == 0 && (batch == 1 || residual_batch_stride % 16 == 0)));
  a.withhold = g_withhold_next_conv.exchange(false) ? 1 : 0;

  ConvMaps maps;
  {  // input: (16 channels, w, h, c1, image), boxes of 16 x (wt, ht) pixels at the conv stride x blocks
    const cuuint64_t dims[5] = {16, (cuuint64_t)gw, (cuuint64_t)gh, (cuuint64_t)c1, (cuuint64_t)batch};
    const cuuint64_t str[4] = {32, (cuuint64_t)gw * 32, (cuuint64_t)(gh * gw * 32),
                               batch > 1 ? (cuuint64_t)x_batch_stride * 2 : 16};  // bytes: dims 1..4
    const cuuint32_t box[5] = {16, (cuuint32_t)(a.halo ? kHaloW : a.wt * stride),
                               (cuuint32_t)(a.halo ? a.sub * a.ht + 2 : a.ht * stride), (cuuint32_t)a.blocks, 1};
    const cuuint32_t unit[5] = {1, (cuuint32_t)stride, (cuuint32_t)stride, 1, 1};
    const CUresult r = encode(&maps.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<void*>(x), dims, str, box, unit,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TTN_UNSUPPORTED, "%s: input tensor map: cuTensorMapEncodeTiled %d", name, (int)r);
  }
  {  // packed weights: (16 channels, co64, tap, c1), boxes of 16 x tile_n x 1 x blocks
    const int taps = kernel * kernel;
    const cuuint64_t dims[4] = {16, (cuuint64_t)co_pad, (cuuint64_t)taps, (cuuint64_t)c1};
    const cuuint64_t str[3] = {32, (cuuint64_t)(co_pad * 32), (cuuint64_t)(taps * co_pad * 32)};
    const cuuint32_t box[4] = {16, (cuuint32_t)a.tile_n, (cuuint32_t)(a.halo ? 9 : 1), (cuuint32_t)a.blocks};
    const cuuint32_t unit[4] = {1, 1, 1, 1};
    const CUresult r = encode(&maps.w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(packed_weights), dims,
                              str, box, unit, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(TTN_UNSUPPORTED, "%s: weight tensor map: cuTensorMapEncodeTiled %d", name, (int)r);
  }
  const size_t stage = a.stage_bytes;
  const void* kernel_fn = residual ? (const void*)conv_tc<true> : (const void*)conv_tc<false>;
  cudaFuncAttributes attr;
  TTN_TRY(cuda_check(cudaFuncGetAttributes(&attr, kernel_fn), "cudaFuncGetAttributes"));
  const int64_t budget = (int64_t)max_dynamic_smem() - (int64_t)attr.sharedSizeBytes - 1024;  // 1 KB: alignment
  a.stages = (int)(budget / (int64_t)stage < kConvMaxStages ? budget / (int64_t)stage : kConvMaxStages);
  if (a.stages < 2) return fail(TTN_UNSUPPORTED, "%s: a ring stage of %zu bytes does not fit twice", name, stage);
  const size_t smem = stage * a.stages + 1024;
  TTN_TRY(ensure_dynamic_smem(kernel_fn, (int)smem));
  const int64_t grid = a.tiles < sm_count() ? a.tiles : sm_count();
  if (residual)
    conv_tc<true><<<(unsigned)grid, kConvThreads, smem, (cudaStream_t)stream>>>(a, maps);
  else
    conv_tc<false><<<(unsigned)grid, kConvThreads, smem, (cudaStream_t)stream>>>(a, maps);
  return launch_check(name);
}

}  // namespace

extern "C" {

ttn_status ttn_conv2d_nc1hwc0_f16(const void* x, int64_t batch, int64_t c1, int64_t h, int64_t w,
                                  int64_t x_batch_stride, const void* packed_weights, const void* bias,
                                  int64_t co, int32_t kernel, int32_t stride, uint32_t flags, void* out,
                                  int64_t out_batch_stride, ttn_stream stream) {
  return conv_launch("ttn_conv2d_nc1hwc0_f16", x, batch, c1, h, w, x_batch_stride, packed_weights, bias, co,
                     kernel, stride, flags, nullptr, 0, out, out_batch_stride, stream);
}

ttn_status ttn_conv2d_residual_nc1hwc0_f16(const void* x, int64_t batch, int64_t c1, int64_t h, int64_t w,
                                           int64_t x_batch_stride, const void* packed_weights, const void* bias,
                                           int64_t co, int32_t kernel, int32_t stride, uint32_t flags,
                                           const void* residual, int64_t residual_batch_stride, void* out,
                                           int64_t out_batch_stride, ttn_stream stream) {
  const char* name = "ttn_conv2d_residual_nc1hwc0_f16";
  if (!residual) return fail(TTN_INVALID_ARG, "%s: null residual", name);
  return conv_launch(name, x, batch, c1, h, w, x_batch_stride, packed_weights, bias, co, kernel, stride, flags,
                     residual, residual_batch_stride, out, out_batch_stride, stream);
}

ttn_status ttn_conv2d_pack_weights_f16(const void* weights, int64_t co, int64_t ci, int32_t kernel, void* packed,
                                       ttn_stream stream) {
  const char* name = "ttn_conv2d_pack_weights_f16";
  if (co <= 0 || ci <= 0 || !(kernel == 1 || kernel == 3 || kernel == 6))
    return fail(TTN_INVALID_ARG, "%s: positive co, ci and kernel 1, 3 or 6", name);
  if (!weights || !packed) return fail(TTN_INVALID_ARG, "%s: null pointer", name);
  const int64_t co_pad = (co + 63) / 64 * 64, taps = (int64_t)kernel * kernel;
  const int64_t total = (ci + 15) / 16 * taps * co_pad * 16;
  const int threads = 256;
  const int64_t blocks = (total + threads - 1) / threads < 4096 ? (total + threads - 1) / threads : 4096;
  conv_pack_weights<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(
      (const uint16_t*)weights, (uint16_t*)packed, (int)co, (int)ci, (int)taps, (int)co_pad, total);
  return launch_check(name);
}

void ttn_conv2d_test_withhold_copies(void) { g_withhold_next_conv.store(true); }

ttn_status ttn_conv2d_fault_f16(uint32_t* fault) {
  if (!fault) return fail(TTN_INVALID_ARG, "ttn_conv2d_fault_f16: null output");
  TTN_TRY(cuda_check(cudaMemcpyFromSymbol(fault, g_conv_fault, sizeof(uint32_t)), "ttn_conv2d_fault_f16"));
  const uint32_t zero = 0;
  return cuda_check(cudaMemcpyToSymbol(g_conv_fault, &zero, sizeof(uint32_t)), "ttn_conv2d_fault_f16");
}

}  // extern "C"
