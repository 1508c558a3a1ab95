// Shared helpers for the libttn kernels: status reporting, strided-view
// coalescing, launch sizing and the fp16 rounding rules of PyTorch CPU eager.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <utility>

#include "../../include/ttn.h"

namespace ttn {

// ------------------------------------------------------------------ status

void set_error(const char* fmt, ...);
ttn_status fail(ttn_status status, const char* fmt, ...);

// Turns a CUDA runtime error (or a pending launch error) into TTN_CUDA_ERROR.
inline ttn_status cuda_check(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return TTN_OK;
  return fail(TTN_CUDA_ERROR, "%s: %s", what, cudaGetErrorString(err));
}
inline ttn_status launch_check(const char* what) {
  return cuda_check(cudaGetLastError(), what);
}

#define TTN_TRY(expr)                   \
  do {                                  \
    ttn_status _s = (expr);             \
    if (_s != TTN_OK) return _s;        \
  } while (0)

// Number of SMs of the current device, cached per device.
int sm_count();

// Raise a kernel's dynamic shared-memory limit to at least `bytes` on the
// current device (the default limit is 48 KB less the kernel's static shared
// memory).  Cached per (device, kernel): the CUDA calls only happen the first
// time a kernel is seen or a larger size is needed, so later calls (e.g. inside
// stream capture after a warm-up call) touch no runtime API.
ttn_status ensure_dynamic_smem(const void* kernel, int bytes);

// Largest opt-in dynamic shared memory per block on the current device.
int max_dynamic_smem();

// Fork/join of an independent branch of one op: branch_fork makes the calling
// thread's auxiliary stream for the current device wait for the work already on
// `stream` and returns it; branch_join makes `stream` wait for everything put on
// the auxiliary stream since.  Under stream capture the branch becomes a
// parallel path of the graph.  Every fork must be followed by its join.
ttn_status branch_fork(cudaStream_t stream, cudaStream_t* aux);
ttn_status branch_join(cudaStream_t stream);

// The 65,536-entry fp16 table of SiLU (kind 0) or sigmoid (kind 1) on the
// current device, indexed by input bits and equal to silu_h / sigmoid_h for
// every input; built on `stream` by the first call.
ttn_status unary_table(int kind, cudaStream_t stream, const uint16_t** table);

// SiLU (kind 0) or sigmoid (kind 1), fp16, over a two-level family of rows:
// element (i1, i2, c) of x sits at x + i1*xs1 + i2*xs2 + c, of y likewise, for
// i1 < n1, i2 < n2, c < ncols.  Rows must be 16-byte aligned (x, y 16-byte
// aligned; strides and ncols multiples of 8).  x may equal y.  Bit-equal to
// silu_h / sigmoid_h per element.
ttn_status unary_rows2_f16(int kind, const uint16_t* x, int64_t xs1, int64_t xs2, uint16_t* y,
                           int64_t ys1, int64_t ys2, int64_t n1, int64_t n2, int64_t ncols,
                           cudaStream_t stream);

// Blocks of `kernel` (at `threads` threads, `smem` dynamic bytes) resident per SM
// on the current device, from the occupancy calculator; cached per (device, kernel).
int resident_blocks(const void* kernel, int threads, size_t smem);

// Grid for a grid-stride loop that keeps every block resident (one full wave):
// min(blocks the work needs, SMs x resident blocks per SM).
template <typename Kernel>
inline unsigned resident_grid(Kernel kernel, int threads, size_t smem, int64_t work,
                              int64_t per_block) {
  int64_t need = (work + per_block - 1) / per_block;
  int64_t cap = (int64_t)sm_count() * resident_blocks((const void*)kernel, threads, smem);
  if (need > cap) need = cap;
  return (unsigned)(need < 1 ? 1 : need);
}

// Grid size for a grid-stride loop: enough blocks for `work` units of `per_block`,
// capped at `waves` resident blocks per SM.
inline unsigned grid_for(int64_t work, int64_t per_block, int waves = 8) {
  int64_t blocks = (work + per_block - 1) / per_block;
  int64_t cap = (int64_t)sm_count() * waves;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (unsigned)blocks;
}

inline size_t dtype_size(int dtype) { return dtype == TTN_F32 ? 4 : 2; }

// ------------------------------------------------------------ view helpers

// A view reduced to its minimal number of dims (size-1 dims dropped, adjacent
// dims merged where every participating view is contiguous across them).
// Dims are stored innermost-first.
struct Coalesced {
  int ndim = 0;
  int64_t size[TTN_MAX_DIMS];
  int64_t stride[4][TTN_MAX_DIMS];  // per operand
  int64_t numel = 1;
};

ttn_status validate(const ttn_tensor* t, const char* name);
bool same_sizes(const ttn_tensor* a, const ttn_tensor* b);
int64_t numel(const ttn_tensor* t);
// Coalesce up to 4 equally-sized views into one iteration space.
Coalesced coalesce(const ttn_tensor* const* views, int count);
// True when the view is dense row-major (C-contiguous) from its data pointer.
bool is_contiguous(const ttn_tensor* t);

// n / d for 32-bit n and a runtime divisor d >= 1 by one multiply-high: with
// l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1 (which fits 32 bits),
// floor(n / d) = (mulhi(n, m) + n) >> l for every n < 2^32 (Granlund and
// Montgomery, "Division by invariant integers using multiplication", 1994).
struct FastDiv {
  uint32_t d, m, l;
  FastDiv() = default;
  explicit FastDiv(uint32_t divisor) : d(divisor), m(0), l(0) {
    while ((1ull << l) < d) ++l;
    m = (uint32_t)((((1ull << 32) * ((1ull << l) - d)) / d) + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    return (uint32_t)(((uint64_t)__umulhi(n, m) + n) >> l);
  }
};

// Device-side iteration space for up to 6 coalesced dims and 3 operands.
struct Index6 {
  int ndim;
  int64_t size[6];
  int64_t stride[3][6];
};

__device__ __forceinline__ void offsets3(const Index6& ix, int64_t linear, int64_t& o0,
                                         int64_t& o1, int64_t& o2) {
  o0 = o1 = o2 = 0;
#pragma unroll
  for (int d = 0; d < 6; ++d) {
    if (d >= ix.ndim) break;
    int64_t q = linear / ix.size[d];
    int64_t r = linear - q * ix.size[d];
    linear = q;
    o0 += r * ix.stride[0][d];
    o1 += r * ix.stride[1][d];
    o2 += r * ix.stride[2][d];
  }
}

// -------------------------------------------------------- fp16 bit helpers

__device__ __forceinline__ uint16_t hbits(__half h) { return __half_as_ushort(h); }
__device__ __forceinline__ __half hfrom(uint16_t b) { return __ushort_as_half(b); }
__device__ __forceinline__ bool hnan_bits(uint16_t b) { return (b & 0x7fffu) > 0x7c00u; }
__device__ __forceinline__ uint16_t hquiet(uint16_t b) { return (uint16_t)(b | 0x0200u); }

// Exact fp16 -> fp32 widening done on bits (keeps NaN sign/payload, quiets it),
// the reference's float_bits (selection_flow.cpp:37-51).
__host__ __device__ __forceinline__ uint32_t float_bits_of_half(uint32_t h) {
  uint32_t sign = (h & 0x8000u) << 16;
  uint32_t exponent = (h >> 10) & 31u;
  uint32_t mantissa = h & 1023u;
  if (exponent == 31u)
    return sign | 0x7f800000u | (mantissa << 13) | (mantissa ? 0x00400000u : 0u);
  if (exponent) return sign | ((exponent + 112u) << 23) | (mantissa << 13);
  if (!mantissa) return sign;
  exponent = 113u;
  while (!(mantissa & 1024u)) {
    mantissa <<= 1;
    --exponent;
  }
  return sign | (exponent << 23) | ((mantissa & 1023u) << 13);
}

// True when r sits within ~8 fp32 ulps of the midpoint between the two fp16
// values around it, i.e. when a few-ulp difference in an fp32 intermediate
// could flip the final fp16 rounding.
__device__ __forceinline__ bool near_half_midpoint(float r) {
  float lo = __half2float(__float2half_rd(r));
  float hi = __half2float(__float2half_ru(r));
  if (!(lo < hi)) return false;  // exactly representable, inf or NaN
  float mid = 0.5f * (lo + hi);  // exact: one more bit than fp16 needs
  return fabsf(r - mid) <= fabsf(r) * 9.5367431640625e-07f;  // 2^-20
}

// fp32 exp(-x) correctly rounded: exp in double, then one rounding to fp32.
__device__ __forceinline__ float exp_neg_cr(float x) { return (float)exp(-(double)x); }

// --- PyTorch CPU eager rules for fp16 unary ops (FP32 math, one rounding) ---
// CPU computes 1/(1+exp(-x)) and x/(1+exp(-x)) in fp32 with IEEE add/div and
// rounds once to fp16.  The GPU uses expf and, when the fp32 result lies near an
// fp16 rounding midpoint, recomputes with a correctly rounded exp so both sides
// round the same fp32 value.  NaN handling follows x86: sigmoid returns the
// quieted -x NaN, silu the quieted x NaN, and silu(-inf) is the default NaN.

__device__ __forceinline__ float sigmoid_f32(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
}
__device__ __forceinline__ float silu_f32(float x) {
  return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}

__device__ __forceinline__ uint16_t sigmoid_h(uint16_t xb) {
  if (hnan_bits(xb)) return hquiet((uint16_t)(xb ^ 0x8000u));
  float x = __half2float(hfrom(xb));
  float r = sigmoid_f32(x);
  if (near_half_midpoint(r)) r = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_neg_cr(x)));
  return hbits(__float2half_rn(r));
}

__device__ __forceinline__ uint16_t silu_h(uint16_t xb) {
  if (hnan_bits(xb)) return hquiet(xb);
  if (xb == 0xfc00u) return 0xfe00u;  // -inf / (1 + inf): x86 default NaN
  float x = __half2float(hfrom(xb));
  float r = silu_f32(x);
  if (near_half_midpoint(r)) r = __fdiv_rn(x, __fadd_rn(1.0f, exp_neg_cr(x)));
  return hbits(__float2half_rn(r));
}

// --- fast path for the same functions on fp16 inputs ---
// ex2.approx / rcp.approx give r within ~12 fp32 ulps of the exact value.  When
// r lands in the fp16 normal range more than 16 fp32 ulps (of the 13 bits that
// fp16 drops) away from a rounding midpoint, CPU's fp32 result (within ~2 ulps
// of exact) rounds to the same fp16 value, so r is final; otherwise (about 0.4%
// of inputs, plus subnormal/overflow/non-finite cases) the exact routine above
// decides.  Both functions take fp16 inputs only, so the exhaustive 65,536-input
// comparison with CPU eager covers the whole domain.

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// exp(-x) to ~2^-20 relative for |x| <= 25 (ex2.approx of a rounded product).
__device__ __forceinline__ float exp_neg_fast(float x) { return ex2_approx(x * -1.44269504088896341f); }
// exp(x) for softmax-style uses (tolerance-gated outputs).
__device__ __forceinline__ float exp_fast(float x) { return ex2_approx(x * 1.44269504088896341f); }

// True when the fast fp32 result r can be rounded to fp16 directly.
__device__ __forceinline__ bool fast_rounding_safe(float r) {
  uint32_t b = __float_as_uint(r) & 0x7fffffffu;
  bool normal = (b - 0x38800000u) < (0x477fe000u - 0x38800000u);  // 2^-14 <= |r| < 65504
  return normal && ((b - 0x0ff0u) & 0x1fffu) > 0x20u;               // > 16 ulps off the midpoint
}

__device__ __forceinline__ float silu_fast_f32(float x) { return x * rcp_approx(1.0f + exp_neg_fast(x)); }
__device__ __forceinline__ float sigmoid_fast_f32(float x) { return rcp_approx(1.0f + exp_neg_fast(x)); }

// Two fp16 lanes at once, deferring the exact decision: returns the fast fp16
// pair and sets `unsafe` where a lane must come from the exact routine instead.
//
// Fast core: a_i = 1 + 2^(-x_i log2 e) (ex2.approx), and the two reciprocals
// share one rcp.approx: q = 1/(a0 a1), 1/a0 = a1 q, 1/a1 = a0 q; then
// sigmoid = 1/a_i, silu = x_i / a_i.  Relative error of r wherever r can sit
// near an fp16 rounding midpoint (|r| >= 2^-25, so |t| < 30 for the ex2
// argument t = -x log2 e): rounding t costs ln2 |t| 2^-24 < 2^-19.6 (damped by
// e/(1+e) <= 1), ex2.approx ~2^-22, rcp.approx 2^-23, and the 1 + e, a0 a1,
// a_j q and x (a_j q) roundings 2^-24 each: below 2^-19 in all.  The result is
// a deterministic function of the input pair, and the exhaustive test over all
// 2^32 pairs checks it against the CPU for every one.
// Bracket: where r*(1-2^-19) and r*(1+2^-19) round to the same fp16 value, the
// true result lies between them and rounds to it too (rounding is monotonic),
// so that value is the result; otherwise (r within 16-32 fp32 ulps of a
// midpoint, any range) the pair is flagged.
// Also flagged: !(a0 a1 < 2^126) -- a NaN input (NaN propagates into the
// product), -inf (a = inf; its CPU results take the exact routine), and
// products so large that q would leave the normal range.  Every other input,
// +inf included (a = 1: silu inf, sigmoid 1), gives a finite product >= 1 and
// a result of the right kind.
template <bool kSilu>
__device__ __forceinline__ uint32_t unary_h2_deferred(uint32_t packed, bool& unsafe) {
  __half2 h = *reinterpret_cast<__half2*>(&packed);
  float2 f = __half22float2(h);
  const float a0 = 1.0f + exp_neg_fast(f.x);
  const float a1 = 1.0f + exp_neg_fast(f.y);
  const float p = a0 * a1;
  const float q = rcp_approx(p);
  float r0 = a1 * q, r1 = a0 * q;
  if (kSilu) {
    r0 *= f.x;
    r1 *= f.y;
  }
  __half2 up = __floats2half2_rn(r0 * 1.0000019073486328125f, r1 * 1.0000019073486328125f);
  __half2 dn = __floats2half2_rn(r0 * 0.9999980926513671875f, r1 * 0.9999980926513671875f);
  uint32_t uw = *reinterpret_cast<uint32_t*>(&up), dw = *reinterpret_cast<uint32_t*>(&dn);
  unsafe = (uw != dw) | !(p < 8.50705917302346159e+37f);  // 2^126
  return uw;
}

// Two fp16 lanes at once; exact fallback per lane when needed.
template <bool kSilu>
__device__ __forceinline__ uint32_t unary_h2_fast(uint32_t packed) {
  __half2 h = *reinterpret_cast<__half2*>(&packed);
  float2 f = __half22float2(h);
  float r0 = kSilu ? silu_fast_f32(f.x) : sigmoid_fast_f32(f.x);
  float r1 = kSilu ? silu_fast_f32(f.y) : sigmoid_fast_f32(f.y);
  __half2 o = __floats2half2_rn(r0, r1);
  uint32_t out = *reinterpret_cast<uint32_t*>(&o);
  if (!fast_rounding_safe(r0)) {
    uint16_t x0 = (uint16_t)(packed & 0xffffu);
    out = (out & 0xffff0000u) | (kSilu ? silu_h(x0) : sigmoid_h(x0));
  }
  if (!fast_rounding_safe(r1)) {
    uint16_t x1 = (uint16_t)(packed >> 16);
    out = (out & 0x0000ffffu) | ((uint32_t)(kSilu ? silu_h(x1) : sigmoid_h(x1)) << 16);
  }
  return out;
}

__device__ __forceinline__ uint16_t sigmoid_h_fast(uint16_t xb) {
  float x = __half2float(hfrom(xb));
  float r = sigmoid_fast_f32(x);
  if (fast_rounding_safe(r)) return hbits(__float2half_rn(r));
  return sigmoid_h(xb);
}

// fp32 versions for TTN_F32 tensors (no rounding step to protect).
__device__ __forceinline__ float sigmoid_f(float x) { return sigmoid_f32(x); }
__device__ __forceinline__ float silu_f(float x) { return silu_f32(x); }

// 16-byte global -> shared copies tracked by commit/wait groups (LDGSTS): the
// hardware counts completion, so a streaming ring needs no software spin.
// Programmatic dependent launch (kernels started with launch_pdl): a kernel may
// begin while the previous kernel on its stream drains; it lets its own successor
// begin likewise (pdl_trigger), does only work that touches no global memory a
// predecessor writes or reads, then waits until the predecessor grid has
// completed and its writes are visible (pdl_wait) before any such access.  Both
// are no-ops in a launch without the attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Paired fp32 arithmetic (Blackwell f32x2 instructions): one instruction does
// the same IEEE round-to-nearest operation on both halves of a 64-bit pair.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(unsigned long long v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// SiLU of two FP32 values as a packed fp16 pair, rounded exactly as
// fp16(silu_f32(x)) is, or flagged.  Fast core: a_i = 1 + 2^(-x_i log2 e)
// (ex2.approx), one rcp.approx for both lanes: q = 1/(a0 a1), r0 = x0 (a1 q),
// r1 = x1 (a0 q) (a1 q's own error in a1 cancels).  Relative error of r: rounding
// the exponent argument t = -x log2 e (fp32 constant 2^-26.2 off, product rounding
// 2^-24) costs ln2 |t| 1.22 2^-24 = |x| 2^-23.71; ex2.approx 2^-22, rcp.approx
// 2^-23 and four roundings 2^-24: in all under |x| 2^-23.71 + 2^-20.68.  silu_f32
// (expf within 2 ulps, then 1 + e and the IEEE divide) is within 2^-21.42 of the
// true value, and forming the bracket ends costs 2^-24.  So with
//   eps(x) = 2^-19.75 + |x| 2^-23.5   (> 1.1 x the sum of those terms)
// silu_f32's result lies in [r (1 - eps), r (1 + eps)], and when both ends round
// to the same fp16 value it rounds to that value as well (rounding is monotonic).
// The pair is returned as u, the rounded upper ends, with `d` = the rounded lower
// ends: a lane whose halves of u and d differ takes silu_f32 itself.  When a0 a1 is
// not below 2^126 (a NaN, -inf, or a product too large for rcp), d = ~u flags both.
constexpr float kEps0 = 1.1341162462485954e-06f;  // 2^-19.75
constexpr float kEps1 = 8.429369557916289e-08f;   // 2^-23.5
__device__ __forceinline__ uint32_t silu_pair_fast(unsigned long long xx, uint32_t& d) {
  const unsigned long long t = f2_mul(xx, f2_pack(-1.44269504088896341f, -1.44269504088896341f));
  const float2 tt = f2_unpack(t);
  const unsigned long long a = f2_add(f2_pack(ex2_approx(tt.x), ex2_approx(tt.y)), f2_pack(1.0f, 1.0f));
  const float2 aa = f2_unpack(a);
  const float p = aa.x * aa.y, q = rcp_approx(p);
  const unsigned long long r = f2_mul(xx, f2_mul(f2_pack(aa.y, aa.x), f2_pack(q, q)));
  const unsigned long long ax = xx & 0x7fffffff7fffffffull;  // |x0|, |x1|
  const unsigned long long eps = f2_fma(ax, f2_pack(kEps1, kEps1), f2_pack(kEps0, kEps0));
  const unsigned long long neps = f2_fma(ax, f2_pack(-kEps1, -kEps1), f2_pack(-kEps0, -kEps0));
  const float2 up = f2_unpack(f2_fma(r, eps, r)), dn = f2_unpack(f2_fma(r, neps, r));
  const __half2 hu = __floats2half2_rn(up.x, up.y), hd = __floats2half2_rn(dn.x, dn.y);
  const uint32_t u = *reinterpret_cast<const uint32_t*>(&hu);
  d = (p < 8.50705917302346159e+37f) ? *reinterpret_cast<const uint32_t*>(&hd) : ~u;  // 2^126
  return u;
}

}  // namespace ttn
