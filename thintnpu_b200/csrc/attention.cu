// C2PSA attention, fused on the 5th-generation tensor cores (tcgen05 + TMEM):
//   S = q^T k (fp16 x fp16 -> fp32 in TMEM), rounded to fp16 (the matmul output),
//   Z = fp16(S * scale), P = fp16(softmax_j(Z)) (FP32 math),
//   out = v P^T (fp16 x fp16 -> fp32 in TMEM), rounded to fp16,
// the operator chain of the reference's Attention block (whole_blocked.py:91-110:
// q^T @ k, * scale, softmax(dim=-1), v @ attn^T) without writing S or P to HBM.
//
// Layouts, as the reference's split of the qkv conv output gives them: q, k
// [kd, n] and v [hd, n] per head with the token dim contiguous; out [hd, n].
// Work item = (image, head, block of 128 queries).  A persistent CTA of 16 warps
// per SM walks its items; thread 0 issues the tensor-core products and threads
// 32 and 64 the copies, all 16 warps run the softmax and the stores:
//  1. TMA brings q (128 queries x kd), k (kd x n) and v (hd x n) into a
//     two-stage shared-memory ring as boxes of 64 tokens (128 bytes, the
//     128-byte swizzle) by all channels: the UMMA canonical 128-byte-swizzled
//     layouts, q and k MN-major (the next 64 tokens one box further, the next
//     8 channels 1024 bytes further), v K-major (8-channel groups 1024 bytes
//     apart, a K=16 step 32 bytes along the row).  Tokens past n are
//     zero-filled.  Each stage has one barrier for q+k and one for v; threads
//     32 and 64 issue the copies while thread 0 issues item k's output product:
//     item k+2's q and k (item k's score product is done with them) and item
//     k+1's v (item k-1's output product is done with it).
//  2. S = q^T k as M=128 x N<=256 x K=16 tcgen05.mma steps into TMEM columns
//     [0, np); item k+1's product is issued before item k's output stores.  In
//     the prescale order (TTN_ATTENTION_PRESCALE) the warps first round the q
//     tile to fp16(q scale) in shared memory and z is fp16(S).
//  3. Warp w reads TMEM lanes 32(w%4).. (its 32 queries) and every fourth
//     32-column chunk (w/4 picks which).  Pass 1 turns S into packed fp16 z
//     (kept in registers) and the row max; pass 2 turns z into fp32
//     e = 2^(z log2e - max log2e), stored in the chunk's own TMEM columns, and
//     the row sum; pass 3 turns e into packed fp16 P = e / sum, stored in the
//     first 16 of the chunk's columns.  Row max and sum are combined over the
//     four warps of a lane quarter in shared memory.
//  4. out^T = P v^T with A = P read from TMEM (K=16 step s takes the 8 columns
//     at 32(s/2) + 8(s%2)) and B = v from shared memory, into the last hd of the
//     CTA's TMEM columns; the warps store their rows.
// Every wait is bounded (200 ms of wall time): on a timeout the CTA records
// which wait gave up in a device word (ttn_attention_fault_f16: 1 = the score
// product, 2 = the output product, 4 = an operand copy), waits (bounded) for
// its copies in flight, frees its TMEM and returns.  Warp-collective
// tensor-memory loads and stores run on every lane of a warp; only global
// stores are guarded per row.
#include "tcgen05.cuh"

namespace ttn {
namespace {

using namespace tc;

constexpr int kAttnRows = 128;     // queries per item (UMMA M, TMEM lanes)
constexpr int kAttnThreads = 512;  // four warps (column groups) per TMEM lane quarter
constexpr int kGroups = kAttnThreads / 128;
constexpr int kChunksPerWarp = 4;  // 32-column chunks per warp: np <= 512 columns
constexpr int kCopierQK = 32;  // the threads that issue the TMA copies of q+k and of v (lane 0 of
constexpr int kCopierV = 64;   // warps 1 and 2, idle while thread 0 issues the output product)
constexpr int kTmemCols = 512;
constexpr float kLog2e = 1.44269504088896341f;

__device__ uint32_t g_attention_fault;

struct AttnArgs {
  const uint16_t* q;
  const uint16_t* k;
  const uint16_t* v;
  uint16_t* out;
  int64_t q_bs, q_hs, q_cs;  // batch, head and channel strides (elements)
  int64_t k_bs, k_hs, k_cs;
  int64_t v_bs, v_hs, v_cs;
  int64_t o_bs, o_hs, o_cs;
  int n, np, nb, kd, hd, heads, tiles;  // nb = 64-token blocks
  int cols;    // TMEM columns: a power of two >= np + hd
  int stages;  // operand buffers in shared memory (2: the next item loads during this one)
  int64_t items;
  float scale;
};
// Tensor maps over q, k, v as 4-D fp16 tensors (token, channel, head, image), boxes of
// 64 tokens x all channels, 128-byte swizzle.
struct AttnMaps {
  CUtensorMap q, k, v;
};

template <bool kPrescale>  // TTN_ATTENTION_PRESCALE: z = fp16(fp16(q scale)^T k), else fp16(fp16(q^T k) scale)
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_tc(AttnArgs a, const __grid_constant__ AttnMaps maps) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t mbar[6];  // score product, output product, q+k copies x2, v copies x2
  __shared__ uint32_t tmem_base_slot;
  __shared__ float red_max[kGroups][kAttnRows], red_sum[kGroups][kAttnRows];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, group = warp >> 2, row = quarter * 32 + lane;
  const int kd = a.kd, hd = a.hd, np = a.np, n = a.n;
  const int chunks = (np + 31) / 32;  // <= 15 (np <= 480): at most kChunksPerWarp per column group
  // shared-memory operands per stage: boxes of 64 tokens x all channels, 128 bytes
  // per channel (all multiples of 1024 bytes)
  const uint32_t lbo_qk = (uint32_t)kd * 128, box_v = (uint32_t)hd * 128;  // one box of q or k, of v
  const uint32_t q_bytes = 2 * lbo_qk, k_bytes = a.nb * lbo_qk, v_bytes = a.nb * box_v;
  const uint32_t stage_bytes = q_bytes + k_bytes + v_bytes;
  const uint32_t smem0 = ((uint32_t)__cvta_generic_to_shared(smem) + 1023u) & ~1023u;
  const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(&mbar[0]);
  const uint32_t bar1 = (uint32_t)__cvta_generic_to_shared(&mbar[1]);
  const uint32_t qk_full0 = (uint32_t)__cvta_generic_to_shared(&mbar[2]);  // stage st: + 8 st
  const uint32_t v_full0 = (uint32_t)__cvta_generic_to_shared(&mbar[4]);
  const int64_t stride = gridDim.x;
  const int count = a.items > (int64_t)blockIdx.x ? (int)((a.items - blockIdx.x + stride - 1) / stride) : 0;

  // threads kCopierQK, kCopierV: copies of this CTA's item j into stage st; thread 0: waits for
  // them and issues the products.  Counters per barrier: q+k of stage 0, 1; v of stage 0, 1.
  uint32_t fills[4] = {0, 0, 0, 0}, waited[4] = {0, 0, 0, 0};
  auto item_coords = [&](int j, int& t, int& h, int& b) {
    const int64_t item = blockIdx.x + j * stride;
    t = (int)(item % a.tiles);
    const int64_t bh = item / a.tiles;
    h = (int)(bh % a.heads), b = (int)(bh / a.heads);
  };
  auto load_qk = [&](int j, int st) {
    int t, h, b;
    item_coords(j, t, h, b);
    const uint32_t full = qk_full0 + 8 * st, sq = smem0 + st * stage_bytes, sk = sq + q_bytes;
    mbar_expect_tx(full, q_bytes + k_bytes);
    tma_load4(sq, &maps.q, t * kAttnRows, 0, h, b, full);
    tma_load4(sq + lbo_qk, &maps.q, t * kAttnRows + 64, 0, h, b, full);
    for (int blk = 0; blk < a.nb; ++blk) tma_load4(sk + blk * lbo_qk, &maps.k, 64 * blk, 0, h, b, full);
    ++fills[st];
  };
  auto load_v = [&](int j, int st) {
    int t, h, b;
    item_coords(j, t, h, b);
    const uint32_t full = v_full0 + 8 * st, sv = smem0 + st * stage_bytes + q_bytes + k_bytes;
    mbar_expect_tx(full, v_bytes);
    for (int blk = 0; blk < a.nb; ++blk) tma_load4(sv + blk * box_v, &maps.v, 64 * blk, 0, h, b, full);
    ++fills[2 + st];
  };
  // which = 0, 1: q+k of stage 0, 1; 2, 3: v of stage 0, 1 (the four barriers are adjacent)
  auto wait_copies = [&](int which) { return mbar_wait(qk_full0 + 8 * which, waited[which]++ & 1); };
  // prescale order: every thread waits for item jj's q+k copies and rounds its share of
  // the q tile to fp16(q * scale) in place before the score product reads it
  unsigned char* const sbase = smem + (smem0 - (uint32_t)__cvta_generic_to_shared(smem));
  auto prescale_q = [&](int jj) -> bool {
    const int st = a.stages == 2 ? (jj & 1) : 0;
    const uint32_t fill = a.stages == 2 ? (uint32_t)(jj >> 1) : (uint32_t)jj;
    const bool ok = mbar_wait(qk_full0 + 8 * st, fill & 1);
    if (ok) {
      uint4* qv = reinterpret_cast<uint4*>(sbase + st * stage_bytes);
      for (int i = tid; i < (int)(q_bytes / 16); i += kAttnThreads) {
        uint4 w = qv[i];
        uint32_t* h = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(bits_h2(h[e]));
          h[e] = h2_bits(__floats2half2_rn(__fmul_rn(f.x, a.scale), __fmul_rn(f.y, a.scale)));
        }
        qv[i] = w;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
    }
    return __syncthreads_and(ok);
  };
  auto score_product = [&](int st, uint32_t& fault) {
    if (!wait_copies(st)) {
      fault |= 4u;  // no commit: the warps' wait for the product gives up too
      return;
    }
    tc_fence_after();
    const uint32_t sq = smem0 + st * stage_bytes, sk = sq + q_bytes;
    for (int col = 0; col < np; col += 256) {
      const int nc = np - col < 256 ? np - col : 256;
      const uint32_t idesc = umma_idesc(kAttnRows, nc, true, true);
      for (int s = 0; s < kd / 16; ++s)  // K=16 channels = two 1024-byte swizzle atoms
        umma_ss(tmem_base_slot + col, smem_desc(sq + s * 2048, lbo_qk, 1024, kSwizzle128B),
                smem_desc(sk + (col / 64) * lbo_qk + s * 2048, lbo_qk, 1024, kSwizzle128B), idesc, s > 0);
    }
    umma_commit(bar0);
  };

  if (tid == 0) {
    for (int i = 0; i < 6; ++i) mbar_init((uint32_t)__cvta_generic_to_shared(&mbar[i]), 1);
    mbar_init_fence();
  }
  if (warp == 0) tmem_alloc((uint32_t)__cvta_generic_to_shared(&tmem_base_slot), a.cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_slot;
  const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
  const uint32_t ocol = a.cols - hd;  // >= np rounded up to 32
  const __half2 neg_inf2 = bits_h2(0xfc00fc00u);
  uint32_t fault = 0;
  if (tid == kCopierQK && count > 0) {
    load_qk(0, 0);
    if (count > 1 && a.stages == 2) load_qk(1, 1);
  }
  if (tid == kCopierV && count > 0) load_v(0, 0);
  bool run = true;
  if (kPrescale && count > 0 && !prescale_q(0)) {
    run = false;
    fault |= 4u;
  }
  if (tid == 0 && count > 0 && run) score_product(0, fault);

  for (int j = 0; j < count && run; ++j) {
    const int st = a.stages == 2 ? (j & 1) : 0;
    const int64_t item = blockIdx.x + j * stride;
    const int t = (int)(item % a.tiles);
    const int64_t bh = item / a.tiles;
    const int h = (int)(bh % a.heads), b = (int)(bh / a.heads);
    const int i0 = t * kAttnRows;
    const uint32_t sv = smem0 + st * stage_bytes + q_bytes + k_bytes;

    bool ok = mbar_wait(bar0, j & 1);  // S of item j in TMEM columns [0, np)
    if (!ok) fault |= 1u;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();

    // 3. softmax over this warp's chunks c = group + kGroups i; warps whose 32
    //    queries all lie past n skip it
    const bool live = i0 + quarter * 32 < n;
    uint32_t z[kChunksPerWarp][16];  // packed fp16 z of this warp's chunks
    __half2 mx2 = neg_inf2;
    if (live) {
#pragma unroll
      for (int i = 0; i < kChunksPerWarp; ++i) {  // pass 1: S -> z (registers), row max
        const int c = group + kGroups * i;
        if (c < chunks) {
          uint32_t r[32];
          tmem_ld32(lane_addr + c * 32, r);
          const bool tail = c * 32 + 32 > n;
#pragma unroll
          for (int p = 0; p < 16; ++p) {
            const __half2 sh = __floats2half2_rn(__uint_as_float(r[2 * p]), __uint_as_float(r[2 * p + 1]));
            const float2 s = __half22float2(sh);
            __half2 zz = kPrescale ? sh : __floats2half2_rn(__fmul_rn(s.x, a.scale), __fmul_rn(s.y, a.scale));
            if (tail && c * 32 + 2 * p >= n) zz = neg_inf2;  // n is even: a pair is valid or not
            mx2 = __hmax2(mx2, zz);
            z[i][p] = h2_bits(zz);
          }
        }
      }
    }
    red_max[group][row] = fmaxf(__low2float(mx2), __high2float(mx2));
    __syncthreads();
    float m = red_max[0][row];
#pragma unroll
    for (int g = 1; g < kGroups; ++g) m = fmaxf(m, red_max[g][row]);
    const float hi = m * kLog2e;
    float sum = 0.0f;
    if (live) {
#pragma unroll
      for (int i = 0; i < kChunksPerWarp; ++i) {  // pass 2: z -> fp32 e (TMEM), row sum
        const int c = group + kGroups * i;
        if (c < chunks) {
          uint32_t e[32];
#pragma unroll
          for (int p = 0; p < 16; ++p) {
            const float2 zf = __half22float2(bits_h2(z[i][p]));
            const float e0 = ex2_approx(__fmaf_rn(zf.x, kLog2e, -hi));
            const float e1 = ex2_approx(__fmaf_rn(zf.y, kLog2e, -hi));
            sum = __fadd_rn(__fadd_rn(sum, e0), e1);
            e[2 * p] = __float_as_uint(e0);
            e[2 * p + 1] = __float_as_uint(e1);
          }
          tmem_st32(lane_addr + c * 32, e);
        }
      }
    }
    red_sum[group][row] = sum;
    tmem_wait_st();
    __syncthreads();
    float total = red_sum[0][row];
#pragma unroll
    for (int g = 1; g < kGroups; ++g) total = __fadd_rn(total, red_sum[g][row]);
    const float inv = __fdiv_rn(1.0f, total);
    if (live) {
#pragma unroll
      for (int i = 0; i < kChunksPerWarp; ++i) {  // pass 3: e -> packed fp16 P (TMEM)
        const int c = group + kGroups * i;
        if (c < chunks) {
          uint32_t e[32], pp[16];
          tmem_ld32(lane_addr + c * 32, e);
#pragma unroll
          for (int p = 0; p < 16; ++p)
            pp[p] = h2_bits(__floats2half2_rn(__fmul_rn(__uint_as_float(e[2 * p]), inv),
                                              __fmul_rn(__uint_as_float(e[2 * p + 1]), inv)));
          tmem_st16(lane_addr + c * 32, pp);
        }
      }
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // 4. out^T = P v^T into TMEM columns [ocol, ocol + hd)
    if (tid == 0) {
      if (!wait_copies(2 + st)) {
        fault |= 4u;  // no commit on a failed copy: the warps' wait below gives up too
      } else {
        tc_fence_after();
        const uint32_t idesc = umma_idesc(kAttnRows, hd, false, false);
        for (int s = 0; s < np / 16; ++s)  // K=16 tokens: 32 bytes along the 128-byte rows of box s/4
          umma_ts(tmem + ocol, tmem + (uint32_t)(32 * (s / 2) + 8 * (s % 2)),
                  smem_desc(sv + (s / 4) * box_v + (s % 4) * 32, 16, 1024, kSwizzle128B), idesc, s > 0);
        umma_commit(bar1);
      }
    }
    // copies into buffers the tensor cores are done with: item j+2's q+k into this stage, item
    // j+1's v into the other (one stage: item j+1's q+k now, its v after the output product)
    if (tid == kCopierQK && j + (a.stages == 2 ? 2 : 1) < count) load_qk(j + (a.stages == 2 ? 2 : 1), st);
    if (tid == kCopierV && a.stages == 2 && j + 1 < count) load_v(j + 1, st ^ 1);
    ok = mbar_wait(bar1, j & 1);
    if (!ok) fault |= 2u;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();
    // TMEM columns [0, np) are free: start item j+1's scores
    if (a.stages == 1 && tid == kCopierV && j + 1 < count) load_v(j + 1, 0);
    if (kPrescale && j + 1 < count && !prescale_q(j + 1)) {
      fault |= 4u;
      break;
    }
    if (tid == 0 && j + 1 < count) score_product(a.stages == 2 ? st ^ 1 : 0, fault);
    if (live && group < hd / 32) {  // output chunk `group` of this warp's 32 queries
      uint16_t* out = a.out + b * a.o_bs + h * a.o_hs + (int64_t)(group * 32) * a.o_cs + i0 + row;
      uint32_t r[32];
      tmem_ld32(lane_addr + ocol + group * 32, r);
      if (i0 + row < n) {
#pragma unroll
        for (int e = 0; e < 32; ++e) out[(int64_t)e * a.o_cs] = __half_as_ushort(__float2half_rn(__uint_as_float(r[e])));
      }
    }
    tc_fence_before();
  }
  if (tid == kCopierQK || tid == kCopierV) {  // copies in flight after an early exit: wait (bounded)
    for (int which = 0; which < 4; ++which)  // at most one fill per barrier is outstanding
      if (fills[which] && !mbar_wait(qk_full0 + 8 * which, (fills[which] - 1) & 1)) fault |= 4u;
  }
  if (fault) atomicOr(&g_attention_fault, fault);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, a.cols);
  }
}

}  // namespace
}  // namespace ttn

using namespace ttn;

namespace {

// Tensor map over a [batch, heads, channels, tokens] fp16 view (token stride 1) as the
// 4-D tensor (token, channel, head, image), box (64 tokens, box_c channels, 1, 1) with
// the 128-byte swizzle: one box lands as box_c swizzled 128-byte rows.
ttn_status encode_operand(CUtensorMap* map, const void* base, int64_t batch, int64_t heads, int64_t channels,
                          int64_t tokens, const int64_t* strides, int box_c, const char* name) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return fail(TTN_CUDA_ERROR, "%s: cuTensorMapEncodeTiled is not available", name);
  const cuuint64_t dims[4] = {(cuuint64_t)tokens, (cuuint64_t)channels, (cuuint64_t)heads, (cuuint64_t)batch};
  // byte strides of dims 1..3; a dim of extent 1 gets any valid stride
  const cuuint64_t str[3] = {(cuuint64_t)strides[2] * 2, heads > 1 ? (cuuint64_t)strides[1] * 2 : 16,
                             batch > 1 ? (cuuint64_t)strides[0] * 2 : 16};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_c, 1, 1};
  const cuuint32_t unit[4] = {1, 1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, str, box, unit,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TTN_UNSUPPORTED, "%s: cuTensorMapEncodeTiled returned %d", name, (int)r);
  return TTN_OK;
}

}  // namespace

extern "C" {

ttn_status ttn_attention_f16(const void* q, const void* k, const void* v, void* out, int64_t batch,
                             int64_t heads, int64_t tokens, int64_t key_dim, int64_t head_dim,
                             const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                             const int64_t* out_strides, float scale, uint32_t flags, ttn_stream stream) {
  const char* name = "ttn_attention_f16";
  if (batch < 0 || heads < 0 || tokens < 0) return fail(TTN_INVALID_ARG, "%s: negative size", name);
  if (flags & ~TTN_ATTENTION_PRESCALE) return fail(TTN_INVALID_ARG, "%s: unknown flags %u", name, flags);
  if (!batch || !heads || !tokens) return TTN_OK;
  if (!q || !k || !v || !out || !q_strides || !k_strides || !v_strides || !out_strides)
    return fail(TTN_INVALID_ARG, "%s: null pointer", name);
  if (key_dim <= 0 || key_dim % 16 || key_dim > 64 || head_dim <= 0 || head_dim % 32 || head_dim > 128)
    return fail(TTN_UNSUPPORTED, "%s: key_dim must be 16..64 in steps of 16, head_dim 32..128 in steps of 32",
                name);
  const int64_t np = (tokens + 15) / 16 * 16;
  if (tokens % 8 || np + head_dim > kTmemCols)
    return fail(TTN_UNSUPPORTED, "%s: tokens must be a multiple of 8 with tokens + head_dim <= 512", name);
  const int64_t* all[4] = {q_strides, k_strides, v_strides, out_strides};
  const void* ptrs[4] = {q, k, v, out};
  const int64_t extents[3] = {batch, heads, 0};
  for (int t = 0; t < 4; ++t) {
    if (((uintptr_t)ptrs[t] & 15u) || all[t][0] % 8 || all[t][1] % 8 || all[t][2] % 8)
      return fail(TTN_INVALID_ARG, "%s: 16-byte aligned bases and strides that are multiples of 8", name);
    for (int d = 0; d < 3; ++d)
      if (all[t][d] <= 0 && (d == 2 || extents[d] > 1))
        return fail(TTN_INVALID_ARG, "%s: batch, head and channel strides must be positive", name);
  }
  const int64_t nb = (tokens + 63) / 64;  // 64-token boxes of k and v
  const size_t stage = (size_t)(2 + nb) * key_dim * 128 + (size_t)nb * head_dim * 128;
  cudaFuncAttributes attr;
  const void* kernel =
      (flags & TTN_ATTENTION_PRESCALE) ? (const void*)attention_tc<true> : (const void*)attention_tc<false>;
  TTN_TRY(cuda_check(cudaFuncGetAttributes(&attr, kernel), "cudaFuncGetAttributes"));
  const int64_t budget = (int64_t)max_dynamic_smem() - (int64_t)attr.sharedSizeBytes - 1024;  // 1 KB: alignment
  if ((int64_t)stage > budget)
    return fail(TTN_UNSUPPORTED, "%s: needs %zu bytes of shared memory", name, stage);
  if (batch > INT32_MAX || heads > INT32_MAX) return fail(TTN_UNSUPPORTED, "%s: batch or heads beyond 2^31", name);
  AttnArgs a;
  a.stages = (int64_t)(2 * stage) <= budget ? 2 : 1;
  const size_t smem = stage * a.stages + 1024;
  TTN_TRY(ensure_dynamic_smem(kernel, (int)smem));
  a.q = (const uint16_t*)q;
  a.k = (const uint16_t*)k;
  a.v = (const uint16_t*)v;
  a.out = (uint16_t*)out;
  a.q_bs = q_strides[0], a.q_hs = q_strides[1], a.q_cs = q_strides[2];
  a.k_bs = k_strides[0], a.k_hs = k_strides[1], a.k_cs = k_strides[2];
  a.v_bs = v_strides[0], a.v_hs = v_strides[1], a.v_cs = v_strides[2];
  a.o_bs = out_strides[0], a.o_hs = out_strides[1], a.o_cs = out_strides[2];
  a.n = (int)tokens, a.np = (int)np, a.nb = (int)nb, a.kd = (int)key_dim, a.hd = (int)head_dim;
  a.heads = (int)heads;
  a.tiles = (int)((tokens + kAttnRows - 1) / kAttnRows);
  a.items = batch * heads * a.tiles;
  a.cols = 32;
  while (a.cols < np + head_dim) a.cols <<= 1;
  a.scale = scale;
  AttnMaps maps;
  TTN_TRY(encode_operand(&maps.q, q, batch, heads, key_dim, tokens, q_strides, (int)key_dim, name));
  TTN_TRY(encode_operand(&maps.k, k, batch, heads, key_dim, tokens, k_strides, (int)key_dim, name));
  TTN_TRY(encode_operand(&maps.v, v, batch, heads, head_dim, tokens, v_strides, (int)head_dim, name));
  const int64_t grid = a.items < sm_count() ? a.items : sm_count();  // one resident CTA per SM
  if (flags & TTN_ATTENTION_PRESCALE)
    attention_tc<true><<<(unsigned)grid, kAttnThreads, smem, (cudaStream_t)stream>>>(a, maps);
  else
    attention_tc<false><<<(unsigned)grid, kAttnThreads, smem, (cudaStream_t)stream>>>(a, maps);
  return launch_check(name);
}

ttn_status ttn_attention_fault_f16(uint32_t* fault) {
  if (!fault) return fail(TTN_INVALID_ARG, "ttn_attention_fault_f16: null output");
  TTN_TRY(cuda_check(cudaMemcpyFromSymbol(fault, g_attention_fault, sizeof(uint32_t)),
                     "ttn_attention_fault_f16"));
  const uint32_t zero = 0;
  return cuda_check(cudaMemcpyToSymbol(g_attention_fault, &zero, sizeof(uint32_t)), "ttn_attention_fault_f16");
}

}  // extern "C"
