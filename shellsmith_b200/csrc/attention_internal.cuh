// Launchers shared between the attention translation units of libshellcache.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace sc {

// Merges `rows` rows of `nparts` (out, lse) partials (paged_attention.cu): part s
// of row r has its D values at po[r * o_row + s * o_part + d] and its lse at
// pl[r * l_row + s * l_part]; with ctx_len set only the splits a decode wrote
// are read. Writes bf16 out (+ lse_out) or, with `packed`, fp32 [r][D + 1].
void launch_combine(const float* po, const float* pl, size_t o_row, size_t o_part, size_t l_row,
                    size_t l_part, const int32_t* ctx_len, int Hq, int nparts,
                    int pages_per_split, int D, int rows, uint16_t* out, float* lse_out,
                    float* packed, cudaStream_t s);

}  // namespace sc
