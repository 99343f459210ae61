/* Plain-C host of the native bridge, built by tests/test_bridge.py with gcc
 * against the engine's shared library (the reference's equivalent is
 * examples/chronos_wrappers/c/main.c).
 *
 *   bridge_runner <checkpoint dir> <dtype> <compile_mode|-> <prediction_length> <runs>
 *
 * Reads the context as whitespace-separated floats on stdin ("nan" = missing),
 * prints the median forecast of the last run, one value per line with 9
 * significant digits, then "latency_ms <value>". */
#include "cutechronos_bridge.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

int main(int argc, char **argv) {
  if (argc != 6) {
    fprintf(stderr, "usage: %s <dir> <dtype> <compile_mode|-> <prediction_length> <runs>\n", argv[0]);
    return 2;
  }
  const char *compile_mode = strcmp(argv[3], "-") ? argv[3] : NULL;
  const int horizon = atoi(argv[4]), runs = atoi(argv[5]);
  int cap = 1024, n = 0;
  float *ctx = (float *)malloc(sizeof(float) * (size_t)cap);
  float v;
  while (scanf("%f", &v) == 1) {
    if (n == cap) {
      cap *= 2;
      ctx = (float *)realloc(ctx, sizeof(float) * (size_t)cap);
    }
    ctx[n++] = v;
  }
  char err[4096];
  int handle = -1;
  if (cutechronos_init_pipeline(argv[1], "cute", "cuda", argv[2], compile_mode, &handle, err, sizeof(err)) != 0) {
    fprintf(stderr, "init failed: %s\n", err);
    return 1;
  }
  float *out = (float *)malloc(sizeof(float) * (size_t)(horizon > 0 ? horizon : 1));
  int out_len = 0;
  double ms = 0.0;
  for (int r = 0; r < runs; ++r) {
    if (cutechronos_predict_median(handle, ctx, n, horizon, out, horizon, &out_len, &ms, err, sizeof(err)) != 0) {
      fprintf(stderr, "predict failed: %s\n", err);
      return 1;
    }
  }
  for (int i = 0; i < out_len; ++i) printf("%.9g\n", out[i]);
  printf("latency_ms %.6f\n", ms);
  if (cutechronos_destroy_pipeline(handle, err, sizeof(err)) != 0) {
    fprintf(stderr, "destroy failed: %s\n", err);
    return 1;
  }
  free(out);
  free(ctx);
  return 0;
}
