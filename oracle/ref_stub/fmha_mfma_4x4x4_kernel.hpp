/* Stub for the reference's AMD-only MFMA kernel header: the reference host
 * file includes it, but the oracle build only uses the host's CPU math. */
#pragma once
#include <hip/hip_runtime.h>
using bhalf_t = __bf16;
using half_t = _Float16;
template <class... A>
inline void launch_fmha_mfma_4x4x4(A...) {
  throw std::logic_error("reference GPU kernel is not built on this machine");
}
