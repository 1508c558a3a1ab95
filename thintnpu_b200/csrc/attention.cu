// C2PSA attention, fused on the 5th-generation tensor cores (tcgen05 + TMEM):
//   S = q^T k (fp16 x fp16 -> fp32 in TMEM), rounded to fp16 (the matmul output),
//   Z = fp16(S * scale), P = fp16(softmax_j(Z)) (FP32 math),
//   out = v P^T (fp16 x fp16 -> fp32 in TMEM), rounded to fp16,
// the operator chain of the reference's Attention block (whole_blocked.py:91-110:
// q^T @ k, * scale, softmax(dim=-1), v @ attn^T) without writing S or P to HBM.
//
// Layouts, as the reference's split of the qkv conv output gives them: q, k
// [kd, n] and v [hd, n] per head with the token dim contiguous; out [hd, n].
// Work item = (image, head, block of 128 queries).  A persistent CTA of 8 warps
// per SM walks the items; while it computes one, cp.async brings the next
// item's operands into the other half of a two-stage shared-memory ring.
//  1. q (128 queries x kd), k (np x kd) and v (hd x np) land in shared memory in
//     the no-swizzle UMMA canonical layouts (8-row x 16-byte core matrices):
//     q and k MN-major (tokens contiguous), v K-major; np = n rounded up to 16,
//     padding zero-filled by the copies.
//  2. One thread issues S = q^T k as M=128 x N<=256 x K=16 tcgen05.mma steps
//     into TMEM columns [0, np).
//  3. Warp w reads TMEM lanes 32(w%4).. (its 32 queries) and every other
//     32-column chunk (w/4 picks which).  Everything stays in TMEM and in the
//     chunk's own columns, so the two warps on a lane quarter never touch each
//     other's data: pass 1 turns S into packed fp16 z (16 columns) and the
//     row max; pass 2 turns z into fp32 e = 2^(z log2e - max log2e) (32 columns)
//     and the row sum; pass 3 turns e into packed fp16 P = e / sum (16
//     columns).  Row max and sum are combined over the two warps in shared memory.
//  4. One thread issues out^T = P v^T with A = P read from TMEM (K=16 step s
//     takes the 8 columns at 32(s/2) + 8(s%2)) and B = v from shared memory,
//     into the last hd of the CTA's TMEM columns; the warps store the rows.
// Every wait is bounded (200 ms of wall time): on a timeout the CTA records
// which wait gave up in a device word (ttn_attention_fault_f16: 1 = the score
// product, 2 = the output product), drains its copies, frees its TMEM and
// returns.  Warp-collective tensor-memory loads and stores run on every lane of
// a warp; only global stores are guarded per row.
#include "common.cuh"

namespace ttn {
namespace {

constexpr int kAttnRows = 128;     // queries per item (UMMA M, TMEM lanes)
constexpr int kAttnThreads = 256;  // two warps per TMEM lane quarter
constexpr int kTmemCols = 512;
constexpr uint64_t kWaitNs = 200ull * 1000 * 1000;  // give up on a tensor-core wait after 200 ms
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
  int n, np, kd, hd, heads, tiles;
  int cols;    // TMEM columns: a power of two >= np + hd
  int stages;  // operand buffers in shared memory (2: the next item loads during this one)
  int64_t items;
  float scale;
};

// Shared-memory matrix descriptor, no swizzle (tcgen05 "version 1"): start
// address, leading-dimension and stride-dimension byte offsets, each >> 4.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}
// Instruction descriptor: f16 x f16 -> f32, M x N, operand majors (1 = MN-major).
__device__ __forceinline__ uint32_t umma_idesc(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}
// D (TMEM) [+]= A (shared memory) x B (shared memory)
__device__ __forceinline__ void umma_ss(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"((uint32_t)acc));
}
// D (TMEM) [+]= A (TMEM, K-major, two fp16 per column) x B (shared memory)
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"((uint32_t)acc));
}
__device__ __forceinline__ void umma_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
               : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits for phase `phase` of the mbarrier, at most kWaitNs of wall time.
__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t phase) {
  const uint64_t start = global_ns();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(mbar), "r"(phase)
        : "memory");
    if (done) return true;
    if (global_ns() - start > kWaitNs) return false;
  }
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 16-byte cp.async that writes zeros when `valid` is false (source size 0)
__device__ __forceinline__ void cp_async16_zfill(uint32_t saddr, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(gmem), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t b) { return *reinterpret_cast<__half2*>(&b); }

__global__ void __launch_bounds__(kAttnThreads, 1) attention_tc(AttnArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t mbar[2];
  __shared__ uint32_t tmem_base_slot;
  __shared__ float red_max[2][kAttnRows], red_sum[2][kAttnRows];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, group = warp >> 2, row = quarter * 32 + lane;
  const int kd = a.kd, hd = a.hd, np = a.np, n = a.n;
  const int chunks = (np + 31) / 32;
  // shared-memory operands per stage (byte offsets; all multiples of 512)
  const uint32_t q_bytes = kAttnRows * kd * 2, k_bytes = np * kd * 2, v_bytes = hd * np * 2;
  const uint32_t stage_bytes = q_bytes + k_bytes + v_bytes;
  const uint32_t smem0 = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t sbo_qk = (uint32_t)(kd / 8) * 128;  // MN-major: next 8 tokens
  const uint32_t sbo_v = (uint32_t)(np / 8) * 128;   // K-major: next 8 channels
  const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(&mbar[0]);
  const uint32_t bar1 = (uint32_t)__cvta_generic_to_shared(&mbar[1]);

  // copies of one item's operands (16-byte chunks of 8 consecutive tokens) into stage `st`
  auto load_item = [&](int64_t item, int st) {
    const int t = (int)(item % a.tiles);
    const int64_t bh = item / a.tiles;
    const int h = (int)(bh % a.heads), b = (int)(bh / a.heads);
    const int i0 = t * kAttnRows;
    const uint16_t* q = a.q + b * a.q_bs + h * a.q_hs;
    const uint16_t* k = a.k + b * a.k_bs + h * a.k_hs;
    const uint16_t* v = a.v + b * a.v_bs + h * a.v_hs;
    const uint32_t sq = smem0 + st * stage_bytes, sk = sq + q_bytes, sv = sk + k_bytes;
    for (int c = tid; c < kd * (kAttnRows / 8); c += kAttnThreads) {  // q^T block, MN-major
      const int d = c / (kAttnRows / 8), t8 = (c % (kAttnRows / 8)) * 8, i = i0 + t8;
      const bool valid = i < n;
      cp_async16_zfill(sq + (t8 / 8) * sbo_qk + (d / 8) * 128 + (d % 8) * 16, valid ? q + d * a.q_cs + i : q,
                       valid);
    }
    for (int c = tid; c < kd * (np / 8); c += kAttnThreads) {  // k, MN-major
      const int d = c / (np / 8), j8 = (c % (np / 8)) * 8;
      const bool valid = j8 < n;
      cp_async16_zfill(sk + (j8 / 8) * sbo_qk + (d / 8) * 128 + (d % 8) * 16, valid ? k + d * a.k_cs + j8 : k,
                       valid);
    }
    for (int c = tid; c < hd * (np / 8); c += kAttnThreads) {  // v, K-major (K = tokens)
      const int ch = c / (np / 8), j8 = (c % (np / 8)) * 8;
      const bool valid = j8 < n;
      cp_async16_zfill(sv + (ch / 8) * sbo_v + (j8 / 8) * 128 + (ch % 8) * 16, valid ? v + ch * a.v_cs + j8 : v,
                       valid);
    }
  };

  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar1));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  int64_t item = blockIdx.x;
  if (item < a.items) load_item(item, 0);
  cp_async_commit();
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(&tmem_base_slot)),
                 "r"(a.cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_slot;
  const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
  const uint32_t ocol = a.cols - hd;  // >= np rounded up to 32
  uint32_t fault = 0;

  for (int it = 0; item < a.items; ++it, item += gridDim.x) {
    const int st = a.stages == 2 ? (it & 1) : 0;
    const int64_t next = item + gridDim.x;
    if (a.stages == 2) {
      if (next < a.items) load_item(next, st ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // copies -> tensor-core reads
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const int t = (int)(item % a.tiles);
    const int64_t bh = item / a.tiles;
    const int h = (int)(bh % a.heads), b = (int)(bh / a.heads);
    const int i0 = t * kAttnRows;
    const uint32_t sq = smem0 + st * stage_bytes, sk = sq + q_bytes, sv = sk + k_bytes;

    // 2. S = q^T k into TMEM columns [0, np): N chunks of at most 256
    if (tid == 0) {
      for (int col = 0; col < np; col += 256) {
        const int nc = np - col < 256 ? np - col : 256;
        const uint32_t idesc = umma_idesc(kAttnRows, nc, true, true);
        for (int s = 0; s < kd / 16; ++s)
          umma_ss(tmem + col, umma_desc(sq + s * 256, 128, sbo_qk),
                  umma_desc(sk + (col / 8) * sbo_qk + s * 256, 128, sbo_qk), idesc, s > 0);
      }
      umma_commit(bar0);
    }
    bool ok = mbar_wait(bar0, it & 1);
    if (!ok) fault |= 1u;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();

    // 3. softmax over this warp's chunks; warps whose 32 queries all lie past n skip it
    const bool live = i0 + quarter * 32 < n;
    __half2 mx2 = bits_h2(0xfc00fc00u);  // -inf, -inf
    if (live) {
      for (int c = group; c < chunks; c += 2) {  // pass 1: S -> packed z, row max
        uint32_t r[32], z[16];
        tmem_ld32(lane_addr + c * 32, r);
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const float2 s = __half22float2(__floats2half2_rn(__uint_as_float(r[2 * p]), __uint_as_float(r[2 * p + 1])));
          __half2 zz = __floats2half2_rn(__fmul_rn(s.x, a.scale), __fmul_rn(s.y, a.scale));
          if (c * 32 + 2 * p >= n) zz = bits_h2(0xfc00fc00u);  // n is even: a pair is valid or not
          mx2 = __hmax2(mx2, zz);
          z[p] = h2_bits(zz);
        }
        tmem_st16(lane_addr + c * 32, z);
      }
    }
    red_max[group][row] = fmaxf(__low2float(mx2), __high2float(mx2));
    tmem_wait_st();
    __syncthreads();
    const float m = fmaxf(red_max[0][row], red_max[1][row]);
    const float hi = m * kLog2e;
    float sum = 0.0f;
    if (live) {
      for (int c = group; c < chunks; c += 2) {  // pass 2: z -> fp32 e, row sum
        uint32_t z[16], e[32];
        tmem_ld16(lane_addr + c * 32, z);
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const float2 zf = __half22float2(bits_h2(z[p]));
          const float e0 = ex2_approx(__fmaf_rn(zf.x, kLog2e, -hi));
          const float e1 = ex2_approx(__fmaf_rn(zf.y, kLog2e, -hi));
          sum = __fadd_rn(__fadd_rn(sum, e0), e1);
          e[2 * p] = __float_as_uint(e0);
          e[2 * p + 1] = __float_as_uint(e1);
        }
        tmem_st32(lane_addr + c * 32, e);
      }
    }
    red_sum[group][row] = sum;
    tmem_wait_st();
    __syncthreads();
    const float inv = __fdiv_rn(1.0f, __fadd_rn(red_sum[0][row], red_sum[1][row]));
    if (live) {
      for (int c = group; c < chunks; c += 2) {  // pass 3: e -> packed fp16 P
        uint32_t e[32], pp[16];
        tmem_ld32(lane_addr + c * 32, e);
#pragma unroll
        for (int p = 0; p < 16; ++p)
          pp[p] = h2_bits(__floats2half2_rn(__fmul_rn(__uint_as_float(e[2 * p]), inv),
                                            __fmul_rn(__uint_as_float(e[2 * p + 1]), inv)));
        tmem_st16(lane_addr + c * 32, pp);
      }
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // 4. out^T = P v^T into TMEM columns [ocol, ocol + hd)
    if (tid == 0) {
      const uint32_t idesc = umma_idesc(kAttnRows, hd, false, false);
      for (int s = 0; s < np / 16; ++s)
        umma_ts(tmem + ocol, tmem + (uint32_t)(32 * (s / 2) + 8 * (s % 2)), umma_desc(sv + s * 256, 128, sbo_v),
                idesc, s > 0);
      umma_commit(bar1);
    }
    ok = mbar_wait(bar1, it & 1);
    if (!ok) fault |= 2u;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();
    if (a.stages == 1 && next < a.items) {  // the only stage is free once the output product is done
      load_item(next, 0);
      cp_async_commit();
    }
    if (live) {
      uint16_t* out = a.out + b * a.o_bs + h * a.o_hs;
      for (int c = group; c < hd / 32; c += 2) {
        uint32_t r[32];
        tmem_ld32(lane_addr + ocol + c * 32, r);
        if (i0 + row < n) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            out[(int64_t)(c * 32 + e) * a.o_cs + i0 + row] = __half_as_ushort(__float2half_rn(__uint_as_float(r[e])));
        }
      }
    }
    tc_fence_before();
  }
  cp_async_wait<0>();
  if (fault) atomicOr(&g_attention_fault, fault);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.cols));
  }
}

}  // namespace
}  // namespace ttn

using namespace ttn;

extern "C" {

ttn_status ttn_attention_f16(const void* q, const void* k, const void* v, void* out, int64_t batch,
                             int64_t heads, int64_t tokens, int64_t key_dim, int64_t head_dim,
                             const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                             const int64_t* out_strides, float scale, ttn_stream stream) {
  const char* name = "ttn_attention_f16";
  if (batch < 0 || heads < 0 || tokens < 0) return fail(TTN_INVALID_ARG, "%s: negative size", name);
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
  for (int t = 0; t < 4; ++t) {
    if (((uintptr_t)ptrs[t] & 15u) || all[t][0] % 8 || all[t][1] % 8 || all[t][2] % 8)
      return fail(TTN_INVALID_ARG, "%s: 16-byte aligned bases and strides that are multiples of 8", name);
  }
  const size_t stage = (size_t)kAttnRows * key_dim * 2 + (size_t)np * key_dim * 2 + (size_t)head_dim * np * 2;
  cudaFuncAttributes attr;
  TTN_TRY(cuda_check(cudaFuncGetAttributes(&attr, (const void*)attention_tc), "cudaFuncGetAttributes"));
  const int64_t budget = (int64_t)max_dynamic_smem() - (int64_t)attr.sharedSizeBytes;
  if ((int64_t)stage > budget)
    return fail(TTN_UNSUPPORTED, "%s: needs %zu bytes of shared memory", name, stage);
  if (batch > INT32_MAX || heads > INT32_MAX) return fail(TTN_UNSUPPORTED, "%s: batch or heads beyond 2^31", name);
  AttnArgs a;
  a.stages = (int64_t)(2 * stage) <= budget ? 2 : 1;
  const size_t smem = stage * a.stages;
  TTN_TRY(ensure_dynamic_smem((const void*)attention_tc, (int)smem));
  a.q = (const uint16_t*)q;
  a.k = (const uint16_t*)k;
  a.v = (const uint16_t*)v;
  a.out = (uint16_t*)out;
  a.q_bs = q_strides[0], a.q_hs = q_strides[1], a.q_cs = q_strides[2];
  a.k_bs = k_strides[0], a.k_hs = k_strides[1], a.k_cs = k_strides[2];
  a.v_bs = v_strides[0], a.v_hs = v_strides[1], a.v_cs = v_strides[2];
  a.o_bs = out_strides[0], a.o_hs = out_strides[1], a.o_cs = out_strides[2];
  a.n = (int)tokens, a.np = (int)np, a.kd = (int)key_dim, a.hd = (int)head_dim, a.heads = (int)heads;
  a.tiles = (int)((tokens + kAttnRows - 1) / kAttnRows);
  a.items = batch * heads * a.tiles;
  a.cols = 32;
  while (a.cols < np + head_dim) a.cols <<= 1;
  a.scale = scale;
  const int64_t grid = a.items < sm_count() ? a.items : sm_count();  // one resident CTA per SM
  attention_tc<<<(unsigned)grid, kAttnThreads, smem, (cudaStream_t)stream>>>(a);
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
