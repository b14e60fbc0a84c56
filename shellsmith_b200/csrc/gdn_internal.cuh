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
// waits for the kernel before it ahead of any memory access. kStateAhead: a
// programmatic dependent whose state chunks stream in while the kernel before
// it still runs; only valid when that kernel never writes the state rows this
// one reads (the decode front kernel, or another layer's update).
enum class BulkLaunch { kOrdinary, kDependent, kStateAhead };
int gdn_bulk_launch(const char* name, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                    const float* g, const float* beta, float* state, const int32_t* slot,
                    uint16_t* out, int B, int Hk, int Hv, int dv, int num_slots, cudaStream_t s,
                    BulkLaunch mode);

}  // namespace sc
