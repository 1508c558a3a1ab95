/*
 * ttn.h -- C ABI of the ThinTNPU-B200 op-pass library (libttn.so).
 *
 * This header is the drop-in boundary for the fp16 tensor-library hot path that
 * runs between the YOLO convolutions: SiLU/sigmoid, broadcast arithmetic,
 * concat/split, NC1HWC0<->NCHW layout, nearest-2x upsample, max-pool/SPPF,
 * row/DFL softmax with anchor decode, and YOLO26 top-k detection selection.
 *
 * Every entry point
 *   - takes raw device pointers, element sizes/strides as int64_t, and a
 *     cudaStream_t (passed as ttn_stream, the same pointer type);
 *   - enqueues its kernels on that stream and returns without synchronising;
 *   - never throws, never aborts, and reports failures as a ttn_status, with a
 *     human-readable message available from ttn_last_error() on the same
 *     thread;
 *   - allocates no device memory: scratch space is passed in by the caller
 *     (sizes from the matching *_workspace_size function).
 * Each declaration names the reference (maxesisnclaw/ThinTNPU) interface it
 * replaces as file:line.
 */
#ifndef TTN_H
#define TTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without including cuda_runtime.h. */
typedef struct CUstream_st* ttn_stream;

typedef enum ttn_status {
  TTN_OK = 0,
  TTN_INVALID_ARG = 1,       /* a shape, stride, pointer or flag is malformed */
  TTN_UNSUPPORTED = 2,       /* well-formed but outside what the op supports */
  TTN_CUDA_ERROR = 3,        /* a CUDA runtime call or a launch failed */
  TTN_TIMEOUT = 4,           /* a bounded device wait ran out */
  TTN_DEVICE_FAULT_FLAG = 5  /* a kernel raised its device status word */
} ttn_status;

typedef enum ttn_dtype { TTN_F16 = 0, TTN_F32 = 1 } ttn_dtype;

typedef enum ttn_binary_op {
  TTN_SUB = 0, /* x - alpha*y */
  TTN_MUL = 1, /* x * y */
  TTN_DIV = 2, /* x / y */
  TTN_ADD = 3  /* x + alpha*y */
} ttn_binary_op;

typedef enum ttn_layout { TTN_NCHW = 0, TTN_NC1HWC0 = 1 } ttn_layout;

#define TTN_MAX_DIMS 8
#define TTN_C0 16

/* A strided view: data points at element [0,...,0]; strides count elements. */
typedef struct ttn_tensor {
  void* data;
  int32_t ndim;
  int32_t dtype; /* ttn_dtype */
  int64_t sizes[TTN_MAX_DIMS];
  int64_t strides[TTN_MAX_DIMS];
} ttn_tensor;

/* ---------------------------------------------------------------- runtime */

/* Library ABI version (major*10000 + minor*100 + patch). */
int ttn_version(void);

/* Static string for a status code. */
const char* ttn_status_string(ttn_status status);

/* Message of the last failing call on this thread ("" if none). */
const char* ttn_last_error(void);

/* Device memory for callers without their own allocator, the C-side twin of the
 * backend allocator (reference backend.cpp:140-151: aclrtMalloc of the size rounded
 * up to whole 32-byte blocks, aclrtFree): cudaMalloc of the rounded size (at least
 * 256-byte aligned), cudaFree.  0 bytes gives a null pointer; ttn_free(NULL) is a
 * no-op.  Not for use while a stream of the calling thread is being captured. */
ttn_status ttn_malloc(void** ptr, size_t bytes);
ttn_status ttn_free(void* ptr);

/* Page-locked host memory (aclrtMallocHost -> cudaMallocHost), the kind the
 * host-buffer path copies from at full link speed; same rounding. */
ttn_status ttn_malloc_host(void** ptr, size_t bytes);
ttn_status ttn_free_host(void* ptr);

/* One asynchronous copy on `stream` (aclrtMemcpyAsync -> cudaMemcpyAsync);
 * kind: 0 host to device, 1 device to host, 2 device to device. */
typedef enum ttn_copy_kind { TTN_HOST_TO_DEVICE = 0, TTN_DEVICE_TO_HOST = 1, TTN_DEVICE_TO_DEVICE = 2 } ttn_copy_kind;
ttn_status ttn_memcpy_async(void* dst, const void* src, size_t bytes, int kind, ttn_stream stream);

/* Stream capture on caller-owned memory, the C-side twin of
 * thin_backend::RuntimeGraph (reference backend.cpp:62-113):
 * aclmdlRICaptureBegin(THREAD_LOCAL) -> cudaStreamBeginCapture(ThreadLocal),
 * aclmdlRICaptureEnd -> cudaStreamEndCapture + cudaGraphInstantiate,
 * aclmdlRIExecuteAsync -> cudaGraphLaunch, aclmdlRIDestroy -> destroy.
 * A graph stays bound to the stream it was begun on and to the creating thread. */
typedef struct ttn_graph ttn_graph;
ttn_status ttn_graph_create(ttn_graph** graph);
ttn_status ttn_graph_begin(ttn_graph* graph, ttn_stream stream);
ttn_status ttn_graph_end(ttn_graph* graph);
ttn_status ttn_graph_replay(ttn_graph* graph);
ttn_status ttn_graph_close(ttn_graph* graph);   /* idempotent */
void ttn_graph_destroy(ttn_graph* graph);       /* closes, then frees the handle */

/* ---------------------------------------------------- elementwise (a1-a3) */

/* y = x / (1 + exp(-x)), FP32 math, one rounding; y may alias x (in place).
 * Replaces silu_impl elementwise.cpp:47-102 and thin_ops::silu_ ops.cpp:498-512;
 * aten::silu aten_adapter.cpp:98-105. x and y have equal sizes, any strides. */
ttn_status ttn_silu(const ttn_tensor* x, const ttn_tensor* y, ttn_stream stream);

/* y = 1 / (1 + exp(-x)), FP32 math, one rounding (bit-equal to CPU eager).
 * Replaces sigmoid_impl sigmoid.cpp:6-44, thin::sigmoid backend.cpp:226-244. */
ttn_status ttn_sigmoid(const ttn_tensor* x, const ttn_tensor* y, ttn_stream stream);

/* out = x (op) alpha*y over equal-sized views; broadcast is a stride of 0.
 * Replaces binary_impl elementwise.cpp:6-45, strided_binary::launch
 * strided_binary.h:192-222 and its dispatch binary() ops.cpp:464-497. */
ttn_status ttn_binary(int op, float alpha, const ttn_tensor* x, const ttn_tensor* y,
                      const ttn_tensor* out, ttn_stream stream);

/* out = a + SiLU(raw) over equal-sized fp16 views that are rows of 16-byte aligned
 * contiguous vectors (e.g. NC1HWC0 images, channel-block slices): SiLU of raw
 * rounded to fp16, then the add in FP32 with one rounding -- bit-identical to
 * ttn_silu followed by ttn_binary(TTN_ADD).  The C2f bottleneck's activation and
 * residual add (silu_ ops.cpp:498-512 on the conv output, then
 * y.append(y[-1] + value) blocked_c2f.py:20-24) without the activation's round
 * trip through HBM.  TTN_UNSUPPORTED for other layouts. */
ttn_status ttn_add_silu_f16(const ttn_tensor* a, const ttn_tensor* raw, const ttn_tensor* out,
                            ttn_stream stream);

/* out = x (op) scalar, the scalar rounded to FP32 first (CPU eager "tensor op
 * python number").  Replaces the fp16 scale multiply whole_blocked.py:101-102. */
ttn_status ttn_binary_scalar(int op, double scalar, const ttn_tensor* x,
                             const ttn_tensor* out, ttn_stream stream);

/* Fused y = SiLU(x + b[c]) + r over NC1HWC0 fp16 [n, c1, hw, 16], FP32 math,
 * one rounding; b is fp16 [c1*16].  The SiLU epilogue of conv_flow.cpp:57-84
 * plus the Bottleneck residual add (ops.cpp:464-493) in one pass. */
ttn_status ttn_bias_silu_residual_nc1hwc0_f16(const void* x, const void* bias,
                                              const void* residual, void* y, int64_t n,
                                              int64_t c1, int64_t hw, ttn_stream stream);

/* ------------------------------------------------ data movement (a4, a5) */

/* dst = src elementwise copy between equal-sized views of the same dtype.
 * Replaces thin_ops::copy_strided ops.cpp:31-84 / materialize::copy
 * ops.cpp:245-288 (device-to-device). */
ttn_status ttn_copy(const ttn_tensor* src, const ttn_tensor* dst, ttn_stream stream);

/* out = cat(inputs, dim).  Inputs of numel 0 are skipped; out must have the
 * concatenated sizes.  Replaces cat() ops.cpp:419-462 with its three paths
 * concatenate::copy :383-416, strided_concat::launch strided_concat.h:163-238
 * and the copy_strided fallback. */
ttn_status ttn_cat(int32_t count, const ttn_tensor* inputs, int32_t dim,
                   const ttn_tensor* out, ttn_stream stream);

/* NC1HWC0 [n, c1, hw, 16] -> NCHW.  Channel c < channels of image b, pixel p
 * goes to y[b*y_batch_stride + c*y_channel_stride + p]; channels <= c1*16 drops
 * the zero-padded tail channels.  Replaces unpack layout_blocked.h:60-69 and the
 * Detect-terminal NCHW restore conv_flow.cpp:87-121 / trim_output :375-403. */
ttn_status ttn_nc1hwc0_to_nchw_f16(const void* x, int64_t n, int64_t c1, int64_t hw,
                                   int64_t channels, void* y, int64_t y_batch_stride,
                                   int64_t y_channel_stride, ttn_stream stream);

/* NCHW [n, channels, hw] -> NC1HWC0 [n, ceil(channels/16), hw, 16], padding
 * channels with +0.  Replaces pack layout_blocked.h:43-58 and
 * pack_input_channels conv_flow.cpp:406-458. */
ttn_status ttn_nchw_to_nc1hwc0_f16(const void* x, int64_t n, int64_t channels,
                                   int64_t hw, void* y, ttn_stream stream);

/* ------------------------------------------------------- spatial (a6, a7) */

/* Nearest 2x upsample.  NCHW: x [n, c, h, w] -> y [n, c, 2h, 2w];
 * NC1HWC0: x [n, c1, h, w, 16] -> y [n, c1, 2h, 2w, 16] (pass c = c1).
 * Contiguous tensors.  Replaces upsample_impl upsample.cpp:5-132,
 * thin::upsample_nearest2d backend.cpp:266-286 and blocked_flow::upsample
 * flow_ops.cpp:233-252. */
ttn_status ttn_upsample2x(int layout, int dtype, const void* x, void* y, int64_t n,
                          int64_t c, int64_t h, int64_t w, ttn_stream stream);

/* Nearest 2x upsample of NC1HWC0 fp16 images that sit at batch strides
 * (elements, multiples of 8) inside larger buffers -- e.g. writing straight into
 * the neck concat's slice (whole_blocked.py:67-68 upsample, then ops.cpp:419
 * cat, with the copy elided).  Image layout [c1, h, w, 16] -> [c1, 2h, 2w, 16]. */
ttn_status ttn_upsample2x_nc1hwc0_f16(const void* x, int64_t x_batch_stride, void* y,
                                      int64_t y_batch_stride, int64_t n, int64_t c1, int64_t h,
                                      int64_t w, ttn_stream stream);

/* kernel x kernel, stride 1, padding kernel/2 max-pool with -inf padding,
 * NaN-propagating (CPU F.max_pool2d semantics).  kernel odd, >= 1.
 * Layouts as ttn_upsample2x.  Replaces maxpool_impl maxpool.cpp:5-191,
 * thin::maxpool2d backend.cpp:245-265, blocked_flow::maxpool flow_ops.cpp:208-231. */
ttn_status ttn_maxpool(int layout, int dtype, int32_t kernel, const void* x, void* y,
                       int64_t n, int64_t c, int64_t h, int64_t w, ttn_stream stream);

/* SPPF tail fused: out = cat(x, p1, p2, p3) along C1 with p(i+1) = maxpool(p(i)),
 * x NC1HWC0 fp16 [n, c1, h, w, 16], out [n, 4*c1, h, w, 16].  Replaces three
 * blocked_flow::maxpool calls plus cat (whole_blocked.py:63-64, ops.cpp:419). */
ttn_status ttn_sppf_f16(const void* x, void* out, int64_t n, int64_t c1, int64_t h,
                        int64_t w, int32_t kernel, ttn_stream stream);

/* --------------------------------------------------------- softmax (a8, a9) */

/* y = softmax(x * scale, dim) over views of equal sizes.  x: f16 or f32;
 * y: same dtype or f32 (half_to_float).  scale != 1 first rounds x*scale to
 * x's dtype (the separate fp16 multiply of whole_blocked.py:101-102).  FP32
 * internals.  Replaces thin_softmax::softmax softmax_host.cpp:51-89 and the
 * kernels Softmax softmax.cpp:6-173 / DflSoftmax :175-271. */
ttn_status ttn_softmax(const ttn_tensor* x, int32_t dim, float scale, const ttn_tensor* y,
                       ttn_stream stream);

/* Fused C2PSA attention (the next step either side of the row softmax):
 * out = v @ softmax(Z)^T per (image, head) with Z = fp16(fp16(q^T @ k) * scale)
 * (YOLO11 order), or with TTN_ATTENTION_PRESCALE Z = fp16(fp16(q * scale)^T @ k)
 * (the YOLO26 order: the query is scaled and rounded before the product).
 * q, k: fp16 [key_dim, tokens] and v, out: fp16 [head_dim, tokens] per head,
 * token dim contiguous; element (b, h, c, t) of each at
 * ptr[b*strides[0] + h*strides[1] + c*strides[2] + t].  The probabilities are
 * rounded to fp16 as the softmax op stores them; both products accumulate in
 * FP32 on the tensor cores (tcgen05, TMEM) and round once to fp16.  Replaces
 * the chain of attention_forward whole_blocked.py:91-103 (both branches of
 * _thin_attention_prescale: channel_select * scale or layout_bmm * scale, then
 * softmax, then the second layout_bmm; layout_bmm/channel_select
 * bmm_flow.cpp:256-358 around thin_softmax::softmax softmax_host.cpp:51-89).
 * key_dim: 16..64 in steps of 16; head_dim: 32..128 in steps of 32; tokens a
 * multiple of 8 with tokens + head_dim <= 512; 16-byte aligned bases, strides
 * positive multiples of 8. */
#define TTN_ATTENTION_PRESCALE 1u
ttn_status ttn_attention_f16(const void* q, const void* k, const void* v, void* out, int64_t batch,
                             int64_t heads, int64_t tokens, int64_t key_dim, int64_t head_dim,
                             const int64_t* q_strides, const int64_t* k_strides,
                             const int64_t* v_strides, const int64_t* out_strides, float scale,
                             uint32_t flags, ttn_stream stream);

/* Reads and clears the attention kernel's fault word: nonzero when a launch
 * gave up waiting for its tensor-core work (it then freed its tensor memory
 * and left its output unwritten).  Synchronous. */
ttn_status ttn_attention_fault_f16(uint32_t* fault);

/* Dense 2-D convolution with the reference's fused epilogue, on the tensor cores
 * (tcgen05 implicit GEMM, FP32 accumulation; a stem-shaped call -- c1 == 1, 3x3
 * stride 2, co <= 64 -- whose weights use input channels past the third runs on the
 * CUDA cores): out = fp16(silu(conv(x, w) + bias)) with TTN_CONV_SILU, else
 * fp16(conv + bias), one rounding.  silu(s) = s / (1 + exp(-s)) evaluated in FP32
 * from exp2 and reciprocal approximations, within ~2^-19 (relative) of the IEEE
 * evaluation, so an output can be the neighbouring fp16 value where that value lies
 * so close to a rounding midpoint (as the FP32 summation order already allows).
 * x: NC1HWC0 fp16 [batch, c1, h, w, 16] (image i at x + i*x_batch_stride; input
 * channels past the real count must be zero, as the reference's pack_input pads).
 * packed_weights: the reference's prepared layout [c1][kernel^2][co64][16] with
 * packed[cb][tap][o][c] = w[o][16 cb + c][tap] (co64 = co rounded up to 64, zero
 * padded; ttn_conv2d_pack_weights_f16 builds it from OIHW).  bias: fp16 [co] or
 * NULL.  kernel 1 (stride 1) or 3 / 6 (stride 1 or 2), zero padding (kernel-1)/2.
 * out: NC1HWC0 [batch, co/16, oh, ow, 16] (co % 16 == 0), or NCHW [batch, co, oh,
 * ow] with TTN_CONV_NCHW, image i at out + i*out_batch_stride (a batch stride
 * larger than one image writes into a concat buffer).  Replaces
 * thin_native_flow::conv conv_flow.cpp:594-646 (kernel convolution_native
 * :123-372, epilogue :45-121) and thin_blocked::conv conv_blocked.cpp. */
#define TTN_CONV_SILU 1u
#define TTN_CONV_NCHW 2u
ttn_status ttn_conv2d_nc1hwc0_f16(const void* x, int64_t batch, int64_t c1, int64_t h, int64_t w,
                                  int64_t x_batch_stride, const void* packed_weights, const void* bias,
                                  int64_t co, int32_t kernel, int32_t stride, uint32_t flags, void* out,
                                  int64_t out_batch_stride, ttn_stream stream);

/* The convolution above with a residual added after its epilogue, as the
 * reference's residual C2f bottleneck does (blocked_c2f.py:20-24: y.append(y[-1] +
 * value), value the cv2 conv's fp16 output): out = fp16(float(residual) +
 * float(y)) with y the fp16 result of ttn_conv2d_nc1hwc0_f16, bit-identical to the
 * conv followed by the separate fp16 add.  residual: NC1HWC0 [batch, co/16, oh,
 * ow, 16], 16-byte aligned, image i at residual + i*residual_batch_stride (a
 * multiple of 8); it may be `out` itself (same pointer and batch stride), any other
 * overlap is undefined.  NC1HWC0 output only (TTN_CONV_NCHW is rejected). */
ttn_status ttn_conv2d_residual_nc1hwc0_f16(const void* x, int64_t batch, int64_t c1, int64_t h, int64_t w,
                                           int64_t x_batch_stride, const void* packed_weights, const void* bias,
                                           int64_t co, int32_t kernel, int32_t stride, uint32_t flags,
                                           const void* residual, int64_t residual_batch_stride, void* out,
                                           int64_t out_batch_stride, ttn_stream stream);

/* Depthwise 2-D convolution (one filter per channel) with the same fused epilogue:
 * acc = sum over (ky, kx) in that order of x * w (FP32, each product and sum rounded),
 * + bias, then silu with TTN_CONV_SILU, one rounding to fp16.  x: NC1HWC0 fp16 [batch,
 * c1, h, w, 16] (image i at x + i*x_batch_stride); packed_weights: [c1][kernel][kernel][16]
 * fp16 (w[c][0][ky][kx] at [c/16][ky][kx][c%16], verify_depthwise_flow.py:27-30);
 * bias: fp16 [16*c1] or NULL; odd kernel 1..7, stride 1 or 2, zero padding kernel/2;
 * out: NC1HWC0 [batch, c1, oh, ow, 16] at out + i*out_batch_stride.  Replaces
 * thin_native_flow::depthwise depthwise_flow.cpp:164-226 (kernel :23-162). */
ttn_status ttn_depthwise_nc1hwc0_f16(const void* x, int64_t batch, int64_t c1, int64_t h, int64_t w,
                                     int64_t x_batch_stride, const void* packed_weights, const void* bias,
                                     int32_t kernel, int32_t stride, uint32_t flags, void* out,
                                     int64_t out_batch_stride, ttn_stream stream);

/* Packs OIHW fp16 weights [co, ci, kernel, kernel] into the layout above
 * (the reference's prepare(), conv_img.cpp:321-383). packed holds
 * ceil(ci/16) * kernel^2 * co64 * 16 elements. */
ttn_status ttn_conv2d_pack_weights_f16(const void* weights, int64_t co, int64_t ci, int32_t kernel,
                                       void* packed, ttn_stream stream);

/* Reads and clears the convolution kernel's fault word: nonzero when a launch
 * gave up waiting (1 = an input copy, 2 = a free ring stage, 4 = an
 * accumulator); its output is then incomplete.  Synchronous. */
ttn_status ttn_conv2d_fault_f16(uint32_t* fault);

/* Test hook for the bounded waits above: the next ttn_conv2d_* launch (from any
 * thread) issues no input copy, so its MMA and epilogue roles wait on barriers
 * that nothing signals; each gives up after its 200 ms limit, sets its bit in the
 * fault word (1 = copy, 4 = accumulator) and the kernel frees its tensor memory
 * and returns with nothing in flight.  The output of that launch is not written.
 * The reference has no counterpart (its kernels do not wait on device flags). */
void ttn_conv2d_test_withhold_copies(void);

/* Fused Detect decode (v8 DFL / v26).  box: fp16 [n, 4*16, a] logits (element
 * (b, s*16+i, j) at box[b*box_bs + (s*16+i)*box_cs + j]); cls: fp16 [n, nc, a]
 * logits with its own strides.  Anchors come from `levels` feature maps of
 * sizes heights[l] x widths[l] with strides[l] (a = sum h*w, grid cell + 0.5).
 * out: fp16 [n, 4+nc, a] contiguous = cat(boxes*stride, sigmoid(cls)), boxes
 * xywh when xywh != 0 else xyxy.  Rounds to fp16 after every step the
 * reference rounds (whole_blocked.py:118-146; DFL softmax.cpp:175-263). */
ttn_status ttn_dfl_decode_f16(const void* box, int64_t box_bs, int64_t box_cs,
                              const void* cls, int64_t cls_bs, int64_t cls_cs, int64_t n,
                              int64_t nc, int32_t levels, const int64_t* heights,
                              const int64_t* widths, const float* strides, int32_t xywh,
                              void* out, ttn_stream stream);

/* ttn_dfl_decode_f16 that also writes the DFL distances it decoded from:
 * distances fp16 [n, 4, a] contiguous (left, top, right, bottom per anchor, each
 * the fp16-rounded expectation of its 16-bin softmax), or NULL to skip.  The
 * reference's chain has this tensor as the output of its DFL (the 1x1 conv with
 * arange(16) weights, whole_blocked.py:138) before the anchor arithmetic of
 * :139-146; tests use it to check the two halves of the decode separately. */
ttn_status ttn_dfl_decode_trace_f16(const void* box, int64_t box_bs, int64_t box_cs,
                                    const void* cls, int64_t cls_bs, int64_t cls_cs, int64_t n,
                                    int64_t nc, int32_t levels, const int64_t* heights,
                                    const int64_t* widths, const float* strides, int32_t xywh,
                                    void* out, void* distances, ttn_stream stream);

/* ------------------------------------------------------- selection (a10) */

/* Flags for ttn_select_f16. */
#define TTN_SELECT_AGNOSTIC 1u     /* one class per anchor (argmax) */
#define TTN_SELECT_NAN_LAST 2u     /* rank NaN scores below -inf (default: above +inf) */
#define TTN_SELECT_SIGMOID 4u      /* decoded[...,4:] are logits: apply fp16 sigmoid first */

/* Optional intermediate outputs, each NULL to skip (the 8 stages of
 * detection_select_trace selection_flow.cpp:385-491). */
typedef struct ttn_select_trace {
  uint16_t* class_max;       /* [b, anchors] best score bits per anchor */
  int64_t* stage1_indices;   /* [b, k] anchors in stage-1 order */
  uint16_t* gathered_scores; /* [b, k, nc] (class-aware only) */
  uint16_t* top_values;      /* [b, k] selected score bits */
  int64_t* stage2_indices;   /* [b, k] flat rank*nc+cls (class-aware only) */
  int64_t* anchor_indices;   /* [b, k] */
  int64_t* labels;           /* [b, k] */
} ttn_select_trace;

/* Bytes of scratch ttn_select_f16 needs (256-byte aligned pointer). */
size_t ttn_select_workspace_size(int64_t batch, int64_t anchors, int64_t classes,
                                 int64_t max_det, uint32_t flags);

/* YOLO26 NMS-free selection over decoded fp16 [b, anchors, 4+nc] (any strides):
 * per-anchor class max, stable top-k anchors, then (class-aware) stable top-k
 * over the k*nc (anchor, class) pairs; writes out FP32 [b, k, 6] rows
 * (x1, y1, x2, y2, score, class), k = min(max_det, anchors).  Order is the
 * reference's total order: score key, then lower index; NaN first.
 * Replaces detection_selection::run selection_flow.cpp:429-491 and
 * thin_native_flow::detection_select :493-514. */
ttn_status ttn_select_f16(const ttn_tensor* decoded, int64_t max_det, uint32_t flags,
                          void* workspace, size_t workspace_bytes, float* out,
                          const ttn_select_trace* trace, ttn_stream stream);

/* Allocation-free variant of ttn_select_f16 for callers that cannot allocate
 * device memory (e.g. bindings that only receive raw device pointers from
 * another runtime, or loops that forbid allocation after start-up).  The scratch
 * lives in an 8 MiB array compiled into the library (held by every GPU that
 * loads it until exit); requests needing more (ttn_select_workspace_size) fail
 * with TTN_UNSUPPORTED.  All calls share that array: calls whose kernels overlap
 * on the GPU race, calls on one stream are safe.  The array's address belongs to
 * the calling thread's current CUDA context and is looked up on every call made
 * outside stream capture (so contexts the host creates itself, or re-creates
 * with cudaDeviceReset, each get theirs); a call under stream capture uses the
 * address found by an earlier call in the same context, and is rejected with
 * TTN_INVALID_ARG when there was none.
 * This entry point has no counterpart in the reference. */
ttn_status ttn_select_f16_static(const ttn_tensor* decoded, int64_t max_det, uint32_t flags,
                                 float* out, const ttn_select_trace* trace, ttn_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* TTN_H */
