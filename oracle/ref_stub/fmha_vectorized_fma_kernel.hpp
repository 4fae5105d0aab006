/* Stub for an AMD-only reference kernel header that the reference host file
 * includes but never launches; the oracle build only uses its CPU math. */
#pragma once
#include <hip/hip_runtime.h>
