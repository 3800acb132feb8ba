// What entry points defined outside hb_engine.cu may read of an engine, and
// the engine's error recording (hb_last_error) for them.
#pragma once

#include <cuda_runtime.h>

#include "hb_internal.h"

namespace hb {

struct EngineView {
  int device;
  cudaStream_t stream;
  int n_sm;
  bool failed;          // a device error ended this engine
  bool uploaded;        // a binned matrix is resident
  bool staged;          // this tree's gradient pairs and scale are resident
  const DevConst* c;
  const uint32_t* fo;   // feature offsets [n_cols + 1]
  const uint8_t* rec;   // row-major records
  const float2* gpair;
  const Scale* scale;
};

void engine_view(const hb_engine* e, EngineView* v);
// Record a device error: the engine refuses every later call.
hb_status engine_fail(hb_engine* e, const char* what, cudaError_t code);
// Record why a call was refused; the engine stays usable.
hb_status engine_refuse(hb_engine* e, const char* why);
// Record why an argument was rejected; returns HB_INVALID_ARGUMENT.
hb_status engine_invalid(hb_engine* e, const char* why);

}  // namespace hb
