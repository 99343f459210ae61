/*
 * cutechronos_bridge.h -- native C bridge of the B200 engine.
 *
 * Same entry points, arguments and error convention as the reference's bridge
 * (examples/chronos_wrappers/include/cutechronos_bridge.h:10-38 of
 * lee101/cutedsl), implemented directly over the C++ engine (include/cc2.h):
 * no embedded Python, no GIL, one handle per loaded model.
 *
 * Every function returns 0 on success and -1 on failure, with a message in
 * error_buffer (NUL-terminated, truncated to error_buffer_size) when given.
 * Unlike the cc2_* entry points, the bridge owns its device memory: the
 * weights, the packed model and the forward workspace of each handle are
 * allocated by cutechronos_init_pipeline / the first predict of a shape and
 * freed by cutechronos_destroy_pipeline.
 */
#ifndef CUTECHRONOS_BRIDGE_H
#define CUTECHRONOS_BRIDGE_H

#include <stddef.h>

#if defined(__GNUC__)
#define CC2_BRIDGE_API __attribute__((visibility("default")))
#else
#define CC2_BRIDGE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Loads a Chronos-2 checkpoint directory (config.json + model.safetensors).
 *   backend      "cute" (or NULL); "original" is not available natively
 *   device       "cuda", "cuda:N" or NULL (= cuda:0); there is no CPU device
 *   dtype_name   "bfloat16" (default) or "float32"
 *   compile_mode NULL/"" = launch the forward's kernels per call; any other
 *                value (e.g. "reduce-overhead") = replay one CUDA graph per
 *                (context length, horizon) shape
 * Reference: cutechronos_bridge.c:96-275 / foreign.py:85-123. */
CC2_BRIDGE_API int cutechronos_init_pipeline(const char *model_id, const char *backend, const char *device,
                                             const char *dtype_name, const char *compile_mode, int *out_handle,
                                             char *error_buffer, size_t error_buffer_size);

/* Median (0.5-quantile) forecast of one series (host float array, NaN =
 * missing) for prediction_length steps into out_values (capacity
 * out_capacity); *out_length = prediction_length; *out_latency_ms = wall
 * time of the call between device synchronisations.
 * Reference: cutechronos_bridge.c:277-385 / foreign.py:140-186. */
CC2_BRIDGE_API int cutechronos_predict_median(int handle, const float *context, int context_length,
                                              int prediction_length, float *out_values, int out_capacity,
                                              int *out_length, double *out_latency_ms, char *error_buffer,
                                              size_t error_buffer_size);

/* Frees the handle's device memory.  Reference: cutechronos_bridge.c:387-406. */
CC2_BRIDGE_API int cutechronos_destroy_pipeline(int handle, char *error_buffer, size_t error_buffer_size);

#ifdef __cplusplus
}
#endif

#endif /* CUTECHRONOS_BRIDGE_H */
