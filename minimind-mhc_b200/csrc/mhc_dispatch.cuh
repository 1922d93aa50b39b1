// Compile-time dispatch helpers: turn runtime (n, dtype, mode) into template
// arguments.  Each helper calls `f` with an std::integral_constant or a dtype
// tag and returns its cudaError_t.
#pragma once

#include <type_traits>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "mhc_b200.h"

namespace mhc {

template <int V> using IC = std::integral_constant<int, V>;

template <typename F>
inline cudaError_t with_n(int n, F &&f) {
  switch (n) {
    case 1: return f(IC<1>{});
    case 2: return f(IC<2>{});
    case 4: return f(IC<4>{});
    case 8: return f(IC<8>{});
    case 16: return f(IC<16>{});
    default: return cudaErrorInvalidValue;
  }
}

template <typename F>
inline cudaError_t with_dtype(int dt, F &&f) {
  switch (dt) {
    case MHC_F32: return f(float{});
    case MHC_BF16: return f(__nv_bfloat16{});
    case MHC_F16: return f(__half{});
    default: return cudaErrorInvalidValue;
  }
}

template <typename F>
inline cudaError_t with_mode(int mode, F &&f) {
  switch (mode) {
    case 0: return f(IC<0>{});
    case 1: return f(IC<1>{});
    case 2: return f(IC<2>{});
    default: return cudaErrorInvalidValue;
  }
}

inline unsigned grid_for(int64_t items, int threads, int sm_count, int per_sm = 16) {
  int64_t b = (items + threads - 1) / threads;
  int64_t cap = (int64_t)(sm_count > 0 ? sm_count : 148) * per_sm;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (unsigned)b;
}

int device_sm_count();

}  // namespace mhc
