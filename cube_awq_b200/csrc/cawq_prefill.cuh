// cawq_prefill.cuh — large-M fused AWQ GEMM on tcgen05 tensor cores (sm_100a).
#pragma once

#include "cawq_common.cuh"

namespace cawq {

bool prefill_supports(const GemmProblem&, const cawq_plan&, const DeviceInfo&) { return false; }

cudaError_t launch_prefill(const GemmProblem&, const cawq_plan&, const DeviceInfo&) {
  return cudaErrorNotSupported;
}

cawq_plan prefill_default_plan(const GemmProblem&, const DeviceInfo&) {
  cawq_plan pl = {};
  pl.path = CAWQ_PATH_PREFILL;
  return pl;
}

void prefill_candidates(const GemmProblem&, const DeviceInfo&, cawq_plan*, int* count, int) {
  *count = 0;
}

}  // namespace cawq
