// cawq_kernels.cu — the device code of libcube_awq.so, one translation unit so
// every kernel shares the device error word without relocatable device code.
#include "cawq_common.cuh"

namespace cawq {

cudaError_t read_device_error(uint32_t* word, int reset) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  e = cudaMemcpyFromSymbol(word, g_cawq_device_error, sizeof(uint32_t));
  if (e != cudaSuccess) return e;
  if (reset) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_cawq_device_error, &zero, sizeof(uint32_t));
  }
  return e;
}

}  // namespace cawq

#include "cawq_decode.cuh"
#include "cawq_dequant.cuh"
#include "cawq_generic.cuh"
#include "cawq_prefill.cuh"
#include "cawq_prefill_f32.cuh"
#include "cawq_prefill_tw.cuh"
#include "cawq_tp.cuh"
