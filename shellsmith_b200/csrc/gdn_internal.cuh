// Launchers shared between the GDN translation units of libshellcache.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace sc {

// The bulk-copy fp32 state update (gdn_decode.cu) handles dk = 128 and dv a
// multiple of 64.
bool gdn_bulk_supported(int dk, int dv);

// Launches it on `s` in one of three ways:
// kOrdinary: a plain launch. kDependent: a programmatic dependent launch that
// waits for the kernel before it ahead of any memory access. kAfterFront: a
// programmatic dependent of the decode front kernel (which writes q/k/v/g/beta
// but never the state), so the state chunks stream in while the front runs.
enum class BulkLaunch { kOrdinary, kDependent, kAfterFront };
int gdn_bulk_launch(const char* name, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                    const float* g, const float* beta, float* state, const int32_t* slot,
                    uint16_t* out, int B, int Hk, int Hv, int dv, int num_slots, cudaStream_t s,
                    BulkLaunch mode);

}  // namespace sc
