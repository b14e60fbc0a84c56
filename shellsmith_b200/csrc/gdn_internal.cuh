// Launchers shared between the GDN translation units of libshellcache.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace sc {

// The bulk-copy fp32 state update (gdn_decode.cu) handles dk = 128 and dv a
// multiple of 64.
bool gdn_bulk_supported(int dk, int dv);

// Launches it; `programmatic` makes it a programmatic dependent of the kernel
// before it on `s`, which must not write the state (the state loads start
// before the kernel waits on its predecessor).
int gdn_bulk_launch(const char* name, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                    const float* g, const float* beta, float* state, const int32_t* slot,
                    uint16_t* out, int B, int Hk, int Hv, int dv, int num_slots, cudaStream_t s,
                    bool programmatic);

}  // namespace sc
