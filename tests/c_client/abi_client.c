/*
 * A plain C host of liboxf.so: it includes only the public headers and
 * calls entry points that need no GPU (version, argument validation with
 * its error string, GEMM descriptor set-up, and a checkpoint v1 write/read
 * round trip of an MLP). It shows the C ABI is usable from C as is, the way
 * an FFI binding from another language would use it. Exit status 0 = pass;
 * otherwise the failing check is printed.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "oxf_host.h"

#define CHECK(cond)                                                    \
  do {                                                                 \
    if (!(cond)) {                                                     \
      fprintf(stderr, "check failed at line %d: %s\n", __LINE__, #cond); \
      return 1;                                                        \
    }                                                                  \
  } while (0)

int main(int argc, char** argv) {
  if (argc != 2) {
    fprintf(stderr, "usage: %s <checkpoint path without extension>\n", argv[0]);
    return 2;
  }
  CHECK(strstr(oxf_version(), "sm_100a") != NULL);

  /* Shape validation happens on the host, before any device work: 10
   * elements cannot be rows of 3 columns. */
  oxf_slice bad = {NULL, 10};
  CHECK(oxf_matrix_softmax_rows(bad, 3, 1.0f, 0, NULL) == OXF_ERR_INVALID_ARG);
  CHECK(strlen(oxf_last_error_string()) > 0);

  /* Descriptor defaults: alpha 1, beta 0, no epilogue, TF32, automatic kernel. */
  oxf_gemm_desc d;
  oxf_gemm_desc_init(&d, 256, 64, 128, 0, 0, NULL, NULL, NULL);
  CHECK(d.M == 256 && d.N == 64 && d.K == 128 && d.batch == 1);
  CHECK(d.alpha == 1.0f && d.beta == 0.0f && d.precision == OXF_PREC_TF32 && d.variant == 0);
  CHECK(d.lda == 128 && d.ldb == 64 && d.ldc == 64);

  /* Checkpoint v1: a 3 -> 5 (GELU) -> 3 MLP with biases and a residual over
   * both layers, written from host arrays and read back. */
  oxf_mlp_spec spec;
  memset(&spec, 0, sizeof(spec));
  spec.n_layers = 2;
  spec.layers[0] = (oxf_layer_spec){3, 5, OXF_ACT_GELU, 1};
  spec.layers[1] = (oxf_layer_spec){5, 3, OXF_ACT_IDENTITY, 1};
  spec.res_start = 0;
  spec.res_end = 2;
  const size_t count = 3 * 5 + 5 + 5 * 3 + 3;
  float params[3 * 5 + 5 + 5 * 3 + 3];
  for (size_t i = 0; i < count; ++i) params[i] = 0.25f * (float)i - 3.0f;
  CHECK(oxf_checkpoint_write_mlp(argv[1], &spec, params, count) == OXF_OK);

  oxf_mlp_spec back;
  float got[3 * 5 + 5 + 5 * 3 + 3];
  size_t n = 0;
  CHECK(oxf_checkpoint_read_mlp(argv[1], &back, NULL, 0, &n) == OXF_OK && n == count);
  CHECK(oxf_checkpoint_read_mlp(argv[1], &back, got, count, &n) == OXF_OK);
  CHECK(memcmp(got, params, sizeof(params)) == 0);
  CHECK(back.n_layers == 2 && back.res_start == 0 && back.res_end == 2);
  CHECK(back.layers[0].in == 3 && back.layers[0].out == 5 && back.layers[0].act == OXF_ACT_GELU &&
        back.layers[0].bias == 1);
  CHECK(back.layers[1].in == 5 && back.layers[1].out == 3 && back.layers[1].bias == 1);
  /* too small a buffer is refused, not overrun */
  CHECK(oxf_checkpoint_read_mlp(argv[1], &back, got, count - 1, &n) != OXF_OK);
  printf("ok\n");
  return 0;
}
