// Quantized matmul entry points (W8A16 per-channel, W4A16 group-128).
#include "runtime.h"

using namespace neso;

extern "C" {

int neso_w8a16_matmul(const void*, const int8_t*, float*, int32_t, int32_t, int32_t, int32_t, int32_t, int32_t,
                      int32_t, uint32_t, uint32_t, uint32_t, neso_stream_t) {
  return fail(NESO_ERR_UNSUPPORTED, "w8a16_matmul: not built yet");
}

int neso_w8a16_scaled_matmul(const void*, const int8_t*, float*, const void*, int32_t, int32_t, int32_t, int32_t,
                             int32_t, int32_t, int32_t, uint32_t, uint32_t, uint32_t, neso_stream_t) {
  return fail(NESO_ERR_UNSUPPORTED, "w8a16_scaled_matmul: not built yet");
}

int neso_w8a16_matmul_mnk(const void*, const int8_t*, const void*, float*, int32_t, int32_t, int32_t,
                          neso_stream_t) {
  return fail(NESO_ERR_UNSUPPORTED, "w8a16_matmul_mnk: not built yet");
}

int neso_w4a16_g128_matmul(const void*, const uint8_t*, const void*, float*, int32_t, int32_t, int32_t,
                           neso_stream_t) {
  return fail(NESO_ERR_UNSUPPORTED, "w4a16_g128_matmul: not built yet");
}

}  // extern "C"
