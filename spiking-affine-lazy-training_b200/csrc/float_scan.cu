// Float chunked affine scan (placeholder until the speculative segment kernel lands).
#include "salt_layers.cuh"

extern "C" salt_status salt_float_fc_scan_workspace_size(int32_t n_out, int32_t n_events,
                                                         size_t* bytes) {
  if (!bytes || n_out < 1 || n_events < 1) return SALT_BAD_ARG;
  *bytes = 256;
  return SALT_OK;
}

extern "C" salt_status salt_float_fc_scan(int32_t, int32_t, int32_t, int32_t, const float*,
                                          const int32_t*, const float*, const float*, float,
                                          float*, int32_t*, int32_t, int32_t*, void*, size_t,
                                          void*) {
  return SALT_BAD_ARG;
}
