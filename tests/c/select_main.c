/* A plain C caller of libttn (no CUDA runtime calls of its own): the selection of
 * INTEGRATION.md's C example on a file of fp16 logits.
 * usage: select_main <in.bin> <out.bin> <b> <a> <nc> <k>
 *   in.bin: fp16 [b, a, 4 + nc] contiguous; out.bin: float [b, min(k, a), 6]. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "ttn.h"

static int select_on_gpu(const uint16_t* decoded_host, int64_t b, int64_t a, int64_t nc, int64_t k,
                         float* out_host) {
  const size_t in_bytes = (size_t)(b * a * (4 + nc)) * 2, out_bytes = (size_t)(b * k * 6) * 4;
  const size_t ws_bytes = ttn_select_workspace_size(b, a, nc, k, TTN_SELECT_SIGMOID);
  void *in = NULL, *out = NULL, *ws = NULL;
  ttn_status s = ttn_malloc(&in, in_bytes);
  if (s == TTN_OK) s = ttn_malloc(&out, out_bytes);
  if (s == TTN_OK) s = ttn_malloc(&ws, ws_bytes);
  if (s == TTN_OK) s = ttn_memcpy_async(in, decoded_host, in_bytes, TTN_HOST_TO_DEVICE, NULL);
  if (s == TTN_OK) {
    ttn_tensor d = {in, 3, TTN_F16, {b, a, 4 + nc}, {a * (4 + nc), 4 + nc, 1}};
    s = ttn_select_f16(&d, k, TTN_SELECT_SIGMOID, ws, ws_bytes, (float*)out, NULL, NULL);
  }
  if (s == TTN_OK) s = ttn_memcpy_async(out_host, out, out_bytes, TTN_DEVICE_TO_HOST, NULL);
  ttn_free(ws);
  ttn_free(out);
  ttn_free(in);
  if (s != TTN_OK) fprintf(stderr, "select: %s\n", ttn_last_error());
  return s;
}

int main(int argc, char** argv) {
  if (argc != 7) {
    fprintf(stderr, "usage: %s in.bin out.bin b a nc k\n", argv[0]);
    return 2;
  }
  const int64_t b = atoll(argv[3]), a = atoll(argv[4]), nc = atoll(argv[5]), max_det = atoll(argv[6]);
  const int64_t k = max_det < a ? max_det : a;
  const size_t in_elems = (size_t)(b * a * (4 + nc)), out_elems = (size_t)(b * k * 6);
  uint16_t* in = malloc(in_elems * 2);
  float* out = malloc(out_elems * 4);
  FILE* f = fopen(argv[1], "rb");
  if (!in || !out || !f || fread(in, 2, in_elems, f) != in_elems) return 3;
  fclose(f);
  const int s = select_on_gpu(in, b, a, nc, k, out);
  if (s != TTN_OK) return 4;
  f = fopen(argv[2], "wb");
  if (!f || fwrite(out, 4, out_elems, f) != out_elems) return 5;
  fclose(f);
  free(in);
  free(out);
  return 0;
}
