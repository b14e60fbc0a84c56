// K7 split-K paged decode attention and the (out, lse) combine.
//
// Reference math: scripts/mlx_attention_qualify.py:234-275 `numpy_attention`
// for one query at the last position (query_offset = keys - 1), GQA head
// j = h // group. Runtime call site: studio_compute/mlx_decode.py:80-106
// `_attention_rows`, which runs mlx-vlm SDPA one request at a time.
//
// B200 mapping.
//   Grid (split, kv head x head group, sequence). A CTA reduces pages
//   [split * pages_per_split, ...) of one sequence for up to 8 query heads
//   that share one kv head, so each K/V byte is read from HBM once per group.
//   Each warp owns NSTAGE shared-memory stages and streams its pages through
//   them with one untiled bulk copy (TMA engine) per page: K and V of one
//   (page, kv head) are one contiguous 2*P*D*2-byte block, pre-swizzled in HBM
//   so ldmatrix reads it without bank conflicts.
//   Scores are computed transposed, S^T[token, head] = K Q^T, with
//   mma.m16n8k16 (M = 16 tokens = one page, N = 8 heads, K = D): no padding
//   rows. The probabilities are transposed in registers with movmatrix into
//   the B operand of O^T[dim, head] += V^T P^T.
//   Online softmax runs in the log2 domain; warps merge in shared memory and
//   the CTA writes a normalised partial and its lse (or the final bf16 output
//   when the sequence needs one split).
#include <math_constants.h>

#include <mutex>

#include "attention_internal.cuh"
#include "common.cuh"
#include "peer.cuh"

namespace sc {
namespace {

constexpr int kPage = 16;
constexpr int kHeadsPerTile = 8;
#ifndef SC_ATTN_QK_ACC
#define SC_ATTN_QK_ACC 2
#endif
constexpr int kQkAcc = SC_ATTN_QK_ACC;  // independent score accumulators per page

template <int D>
struct AttnShape {
  static constexpr int ROW_BYTES = D * 2;
  static constexpr int KV_BYTES = kPage * ROW_BYTES;  // K or V block of one page, one head
  static constexpr int STAGE_BYTES = 2 * KV_BYTES;
  static constexpr int KSTEPS = D / 16;
};

// The most parts the in-kernel merge of the one-launch layer takes; a launch with
// more splits (a few very long sequences) merges in the separate combine kernel,
// whose (row, 32-dim) CTAs spread the reads over the SMs.
constexpr int kFusedMergeParts = 16;

// The last CTA of a (sequence, kv head, head group) to finish merges the
// normalised partials of the sequence's `ns` <= kFusedMergeParts splits for its
// `heads` query heads: out = sum_s e^(lse_s - M) o_s / sum_s e^(lse_s - M). All
// heads at once: warp w makes the weights of heads w, w + NW, ... into shared
// memory `w` ([8][kFusedMergeParts]), then each thread sums float4 column
// groups of every head over the parts, all loads independent. Other CTAs'
// partials are read through L2 (ld.global.cg): L1 is not coherent across SMs.
template <int D, int NW>
__device__ void merge_splits(const float* part_out, const float* part_lse, size_t row0,
                             int heads, int num_splits, int ns, float* w, uint16_t* out,
                             float* lse_out, float* packed) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int h = warp; h < heads; h += NW) {
    const float ls = lane < ns ? __ldcg(part_lse + (row0 + h) * num_splits + lane) : -CUDART_INF_F;
    float m = ls;
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float e = (ls == -CUDART_INF_F) ? 0.f : __expf(ls - m);
    float sum = e;
    for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const bool empty = m == -CUDART_INF_F;
    if (lane < kFusedMergeParts) w[h * kFusedMergeParts + lane] = empty ? 0.f : e / sum;
    if (lane == 0) {
      const float l = empty ? -CUDART_INF_F : m + logf(sum);
      if (packed != nullptr)
        packed[(row0 + h) * (D + 1) + D] = l;
      else if (lse_out != nullptr)
        lse_out[row0 + h] = l;
    }
  }
  __syncthreads();
  constexpr int kGroups = D / 4;  // float4 column groups per head
  for (int g = threadIdx.x; g < heads * kGroups; g += NW * 32) {
    const int h = g / kGroups, c = 4 * (g - h * kGroups);
    const float* po = part_out + (row0 + h) * (size_t)num_splits * D + c;
    const float* wh = w + h * kFusedMergeParts;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int s = 0; s < ns; ++s) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(po + (size_t)s * D));
      const float ws = wh[s];
      acc.x = fmaf(ws, v.x, acc.x);
      acc.y = fmaf(ws, v.y, acc.y);
      acc.z = fmaf(ws, v.z, acc.z);
      acc.w = fmaf(ws, v.w, acc.w);
    }
    const size_t row = row0 + h;
    if (packed != nullptr) {
      float* dst = packed + row * (D + 1) + c;
      dst[0] = acc.x;
      dst[1] = acc.y;
      dst[2] = acc.z;
      dst[3] = acc.w;
    } else {
      uint2 pk;
      pk.x = pack_bf16x2(acc.x, acc.y);
      pk.y = pack_bf16x2(acc.z, acc.w);
      *reinterpret_cast<uint2*>(out + row * D + c) = pk;
    }
  }
}

// What the one-launch attention layer (kFused) adds to the split-K kernel: the
// new token's K/V rows [B][Hkv][D] and their slots (page * 16 + offset, < 0
// skips a row), the pool written through, and, when the splits merge in the
// kernel, one arrival counter per (sequence, kv head, head group), zero between
// launches.
struct FusedArgs {
  const uint16_t* k_new = nullptr;
  const uint16_t* v_new = nullptr;
  const int64_t* slot_mapping = nullptr;
  uint16_t* pool = nullptr;
  unsigned int* counters = nullptr;
  int merge = 0;  // 1: the splits merge in the kernel (num_splits <= kFusedMergeParts)
};

template <int D, int NW, int NSTAGE, bool kFused>
__global__ void __launch_bounds__(NW * 32)
    paged_decode_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ kv_pool,
                        const int32_t* __restrict__ block_table,
                        const int32_t* __restrict__ ctx_len,
                        const int32_t* __restrict__ seq_order, int Hq, int Hkv, int G, int HG,
                        int max_pages, int pages_per_split, int num_splits, float scale_log2,
                        float* __restrict__ part_out, float* __restrict__ part_lse,
                        uint16_t* __restrict__ out, float* __restrict__ lse_out,
                        float* __restrict__ packed, long long num_pages,
                        unsigned int* status, FusedArgs fa) {
  using S = AttnShape<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NW * NSTAGE * S::STAGE_BYTES);
  pdl_wait();
  pdl_trigger();

  const int split = blockIdx.x;
  const int kvh = blockIdx.y / HG;
  const int hg = blockIdx.y - kvh * HG;
  // Sequences in launch order (longest first shortens the tail of ragged batches).
  const int b = seq_order != nullptr ? seq_order[blockIdx.z] : (int)blockIdx.z;
  if (b < 0 || b >= (int)gridDim.z) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) flag_device(status, DEV_BAD_INDEX);
    return;
  }
  const int L = checked_ctx_len(ctx_len[b], kPage, max_pages, pages_per_split, num_splits,
                                status, split == 0 && blockIdx.y == 0 && threadIdx.x == 0);
  const int npages = (L + kPage - 1) / kPage;
  const int p_begin = split * pages_per_split;
  // Splits this sequence fills: with one, the CTA writes the final rows itself.
  const int ns_seq = (npages + pages_per_split - 1) / pages_per_split;
  const bool final_here = num_splits == 1 || (kFused && fa.merge && ns_seq <= 1);

  // The appended token (kFused): its page and offset, and its rows written to
  // the pool once per (sequence, kv head), by split 0 of head group 0. A CTA
  // whose pages include that page replaces the row in its own stage copy, so no
  // CTA depends on when the write lands.
  long long slot_page = -1;
  int slot_off = 0;
  if constexpr (kFused) {
    const int64_t slot = fa.slot_mapping != nullptr ? fa.slot_mapping[b] : -1;
    if (slot >= 0 && slot / kPage < num_pages) {
      slot_page = slot / kPage;
      slot_off = (int)(slot - slot_page * kPage);
    } else if (slot >= 0 && split == 0 && hg == 0 && threadIdx.x == 0) {
      flag_device(status, DEV_BAD_INDEX);
    }
    if (slot_page >= 0 && split == 0 && hg == 0) {
      const uint4* kr = reinterpret_cast<const uint4*>(fa.k_new + ((size_t)b * Hkv + kvh) * D);
      const uint4* vr = reinterpret_cast<const uint4*>(fa.v_new + ((size_t)b * Hkv + kvh) * D);
      for (int c = threadIdx.x; c < 2 * (D / 8); c += blockDim.x) {
        const int which = c / (D / 8), cc = c - which * (D / 8);
        uint16_t* dst = fa.pool + ((((size_t)slot_page * Hkv + kvh) * 2 + which) * kPage +
                                   slot_off) * D + 8 * (cc ^ (slot_off & 7));
        *reinterpret_cast<uint4*>(dst) = which ? vr[cc] : kr[cc];
      }
    }
  }

  // After any bounded wait has given up on this device, later CTAs stop at
  // once instead of each waiting out its own limit (a fused CTA still counts
  // its arrival, so the counters stay consistent for the next launch).
  if (status != nullptr && (*reinterpret_cast<volatile unsigned int*>(status) & DEV_WAIT_TIMEOUT)) {
    if constexpr (kFused) {
      if (fa.merge && !final_here && p_begin < npages && threadIdx.x == 0) {
        unsigned int* ctr = fa.counters + ((size_t)b * Hkv + kvh) * HG + hg;
        if (atomicAdd(ctr, 1u) == (unsigned int)(ns_seq - 1)) *ctr = 0u;
      }
    }
    return;
  }
  if (npages == 0 && split == 0) {  // nothing to attend: zero output, lse = -inf
    for (int idx = threadIdx.x; idx < min(kHeadsPerTile, G - hg * kHeadsPerTile) * D;
         idx += blockDim.x) {
      const size_t row = (size_t)b * Hq + kvh * G + hg * kHeadsPerTile + idx / D;
      if (final_here && packed != nullptr) {
        packed[row * (D + 1) + idx % D] = 0.f;
        if (idx % D == 0) packed[row * (D + 1) + D] = -CUDART_INF_F;
      } else if (final_here) {
        out[row * D + idx % D] = 0;
        if (idx % D == 0 && lse_out != nullptr) lse_out[row] = -CUDART_INF_F;
      }
    }
    return;
  }
  if (p_begin >= npages) return;  // uniform over the CTA
  const int n_here = min(npages, p_begin + pages_per_split) - p_begin;
  const int heads_here = min(kHeadsPerTile, G - hg * kHeadsPerTile);
  const int head0 = kvh * G + hg * kHeadsPerTile;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NW * NSTAGE; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // Q^T as the B operand: b0 = q[n][16kk + 2c .. +1], b1 = q[n][16kk + 8 + 2c .. +1].
  uint32_t qf[S::KSTEPS][2];
  {
    const int n = lane >> 2, c = lane & 3;
    const bool valid = n < heads_here;
    const uint16_t* qp = q + ((size_t)b * Hq + head0 + (valid ? n : 0)) * D;
#pragma unroll
    for (int kk = 0; kk < S::KSTEPS; ++kk) {
      qf[kk][0] = valid ? *reinterpret_cast<const uint32_t*>(qp + 16 * kk + 2 * c) : 0u;
      qf[kk][1] = valid ? *reinterpret_cast<const uint32_t*>(qp + 16 * kk + 8 + 2 * c) : 0u;
    }
  }

  // Pages of this warp: p_begin + warp + j * NW, j < nj.
  const int nj = n_here > warp ? (n_here - warp + NW - 1) / NW : 0;
  uint8_t* stage = smem + warp * NSTAGE * S::STAGE_BYTES;
  uint64_t* bar = bars + warp * NSTAGE;
  const int32_t* bt_row = block_table + (size_t)b * max_pages;

  auto issue = [&](int j) {
    int page = bt_row[p_begin + warp + j * NW];
    if (page < 0 || page >= num_pages) {
      flag_device(status, DEV_BAD_INDEX);
      page = 0;  // keep the copy in bounds; the status word reports the fault
    }
    const uint8_t* src =
        reinterpret_cast<const uint8_t*>(kv_pool) + ((size_t)page * Hkv + kvh) * S::STAGE_BYTES;
    const int s = j % NSTAGE;
    mbar_arrive_expect_tx(&bar[s], S::STAGE_BYTES);
    bulk_g2s(stage + s * S::STAGE_BYTES, src, S::STAGE_BYTES, &bar[s]);
  };

  int issued = 0;
  if (lane == 0)
    for (; issued < NSTAGE && issued < nj; ++issued) issue(issued);
  issued = __shfl_sync(0xffffffffu, issued, 0);

  float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F;  // running max of heads 2c, 2c+1 (log2 units)
  float l0 = 0.f, l1 = 0.f;                      // this lane's partial sums
  float o[S::KSTEPS][4];
#pragma unroll
  for (int mt = 0; mt < S::KSTEPS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

  const int mi = lane >> 3, r8 = lane & 7;
  const int tk = r8 + 8 * (mi & 1);   // token row this lane addresses for K
  const int tv = r8 + 8 * (mi >> 1);  // token row this lane addresses for V^T
  int consumed = 0;
  for (int j = 0; j < nj; ++j) {
    const int s = j % NSTAGE;
    if (!mbar_wait_bounded(&bar[s], (j / NSTAGE) & 1, status)) break;
    const uint32_t kbase = smem_addr(stage + s * S::STAGE_BYTES);
    const uint32_t vbase = kbase + S::KV_BYTES;
    const int page_tok = (p_begin + warp + j * NW) * kPage;
    if (page_tok + kPage > L) {
      // Rows past the context hold whatever the pool held (possibly Inf/NaN
      // bits); their probability is 0, but 0 * Inf would poison the sum.
      uint4* vrows = reinterpret_cast<uint4*>(stage + s * S::STAGE_BYTES + S::KV_BYTES);
      for (int c = (L - page_tok) * (S::ROW_BYTES / 16) + lane; c < kPage * (S::ROW_BYTES / 16);
           c += 32)
        vrows[c] = make_uint4(0u, 0u, 0u, 0u);
      __syncwarp();
    }
    if constexpr (kFused) {
      // The appended token's page: its row in this stage copy comes from the
      // new K/V (the copy may predate the pool write).
      if (slot_page >= 0 && bt_row[p_begin + warp + j * NW] == slot_page) {
        const uint4* kr = reinterpret_cast<const uint4*>(fa.k_new + ((size_t)b * Hkv + kvh) * D);
        const uint4* vr = reinterpret_cast<const uint4*>(fa.v_new + ((size_t)b * Hkv + kvh) * D);
        uint8_t* krow = stage + s * S::STAGE_BYTES + slot_off * S::ROW_BYTES;
        for (int c = lane; c < D / 8; c += 32) {
          const int at = (c ^ (slot_off & 7)) << 4;
          *reinterpret_cast<uint4*>(krow + at) = kr[c];
          *reinterpret_cast<uint4*>(krow + S::KV_BYTES + at) = vr[c];
        }
        __syncwarp();
      }
    }

    // kQkAcc accumulators over the K steps cut the dependent MMA chain of the scores.
    float sca[kQkAcc][4];
#pragma unroll
    for (int x = 0; x < kQkAcc; ++x) sca[x][0] = sca[x][1] = sca[x][2] = sca[x][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < S::KSTEPS; ++kk) {
      const int chunk = 2 * kk + (mi >> 1);
      uint32_t a0, a1, a2, a3;
      ldsm_x4(kbase + tk * S::ROW_BYTES + ((chunk ^ (tk & 7)) << 4), a0, a1, a2, a3);
      mma_bf16_16816(sca[kk % kQkAcc], a0, a1, a2, a3, qf[kk][0], qf[kk][1]);
    }
    float sc4[4] = {sca[0][0], sca[0][1], sca[0][2], sca[0][3]};
#pragma unroll
    for (int x = 1; x < kQkAcc; ++x)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc4[e] += sca[x][e];

    const int tok0 = page_tok + (lane >> 2);
    const bool lo_ok = tok0 < L, hi_ok = tok0 + 8 < L;
    const float x0 = lo_ok ? sc4[0] * scale_log2 : -CUDART_INF_F;
    const float x1 = lo_ok ? sc4[1] * scale_log2 : -CUDART_INF_F;
    const float x2 = hi_ok ? sc4[2] * scale_log2 : -CUDART_INF_F;
    const float x3 = hi_ok ? sc4[3] * scale_log2 : -CUDART_INF_F;
    float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    // The first token of every page is < L, so mx0 / mx1 are finite.
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = exp2f(m0 - mn0), c1 = exp2f(m1 - mn1);
    const float p0 = exp2f(x0 - mn0), p1 = exp2f(x1 - mn1);
    const float p2 = exp2f(x2 - mn0), p3 = exp2f(x3 - mn1);
    l0 = fmaf(l0, c0, p0 + p2);
    l1 = fmaf(l1, c1, p1 + p3);
    m0 = mn0;
    m1 = mn1;
    const uint32_t pb0 = movmatrix_t(pack_bf16x2(p0, p1));
    const uint32_t pb1 = movmatrix_t(pack_bf16x2(p2, p3));
#pragma unroll
    for (int mt = 0; mt < S::KSTEPS; ++mt) {
      o[mt][0] *= c0;
      o[mt][1] *= c1;
      o[mt][2] *= c0;
      o[mt][3] *= c1;
      const int chunk = 2 * mt + (mi & 1);
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(vbase + tv * S::ROW_BYTES + ((chunk ^ (tv & 7)) << 4), a0, a1, a2, a3);
      mma_bf16_16816(o[mt], a0, a1, a2, a3, pb0, pb1);
    }
    consumed = j + 1;
    __syncwarp();
    if (lane == 0 && issued < nj) {
      fence_proxy_async_smem();
      issue(issued);
    }
    if (issued < nj) ++issued;
  }
  if (consumed < nj) {
    // A wait gave up (already flagged): drain this warp's copies in flight so
    // the CTA never exits with a bulk copy still writing its shared memory.
    for (int j = consumed; j < issued; ++j)
      if (!mbar_wait_bounded(&bar[j % NSTAGE], (j / NSTAGE) & 1, status)) break;
  }

#pragma unroll
  for (int off = 4; off <= 16; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  __syncthreads();  // every stage is drained; reuse the stage memory

  float* red_o = reinterpret_cast<float*>(smem);                 // [NW][8][D]
  float* red_m = red_o + NW * kHeadsPerTile * D;                 // [NW][8]
  float* red_l = red_m + NW * kHeadsPerTile;                     // [NW][8]
  {
    const int d0 = lane >> 2, h0 = 2 * (lane & 3);
    float* w0 = red_o + (warp * kHeadsPerTile + h0) * D;
    float* w1 = w0 + D;
#pragma unroll
    for (int mt = 0; mt < S::KSTEPS; ++mt) {
      w0[16 * mt + d0] = o[mt][0];
      w1[16 * mt + d0] = o[mt][1];
      w0[16 * mt + d0 + 8] = o[mt][2];
      w1[16 * mt + d0 + 8] = o[mt][3];
    }
    if (lane < 4) {
      red_m[warp * kHeadsPerTile + h0] = m0;
      red_m[warp * kHeadsPerTile + h0 + 1] = m1;
      red_l[warp * kHeadsPerTile + h0] = l0;
      red_l[warp * kHeadsPerTile + h0 + 1] = l1;
    }
  }
  __syncthreads();

  constexpr float kLn2 = 0.6931471805599453f;
  for (int idx = threadIdx.x; idx < heads_here * D; idx += NW * 32) {
    const int n = idx / D, d = idx - (idx / D) * D;
    float M = -CUDART_INF_F;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, red_m[w * kHeadsPerTile + n]);
    float lsum = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float mw = red_m[w * kHeadsPerTile + n];
      const float f = mw == -CUDART_INF_F ? 0.f : exp2f(mw - M);
      lsum = fmaf(red_l[w * kHeadsPerTile + n], f, lsum);
      acc = fmaf(red_o[(w * kHeadsPerTile + n) * D + d], f, acc);
    }
    const float val = acc / lsum;
    const float lse = (M + log2f(lsum)) * kLn2;
    const size_t row = (size_t)b * Hq + head0 + n;
    if (final_here && packed != nullptr) {
      packed[row * (D + 1) + d] = val;
      if (d == 0) packed[row * (D + 1) + D] = lse;
    } else if (final_here) {
      out[row * D + d] = f_to_bf16(val);
      if (d == 0 && lse_out != nullptr) lse_out[row] = lse;
    } else {
      part_out[(row * num_splits + split) * D + d] = val;
      if (d == 0) part_lse[row * num_splits + split] = lse;
    }
  }
  if constexpr (kFused) {
    // Count this split in; the last of the sequence's splits to arrive merges them
    // (no CTA waits for another) and leaves the counter at zero for the next launch.
    if (fa.merge && !final_here) {
      __shared__ int s_last;
      __syncthreads();  // every thread's partials precede thread 0's release below
      if (threadIdx.x == 0) {
        unsigned int* ctr = fa.counters + ((size_t)b * Hkv + kvh) * HG + hg;
        __threadfence();  // cumulative: the CTA's partials are visible before the count
        const int last = atomicAdd(ctr, 1u) == (unsigned int)(ns_seq - 1);
        if (last) {
          *ctr = 0u;
          __threadfence();  // every other split's partials are visible from here
        }
        s_last = last;
      }
      __syncthreads();
      if (s_last) {
        float* w = reinterpret_cast<float*>(smem);  // the stage memory is free
        merge_splits<D, NW>(part_out, part_lse, (size_t)b * Hq + head0, heads_here,
                            num_splits, ns_seq, w, out, lse_out, packed);
      }
    }
  }
}

// One CTA per output row: merges the partials of that row.
// Part s of row r: value d at po[r * o_row + s * o_part + d], lse at
// pl[r * l_row + s * l_part]. With ctx_len != NULL only the splits the decode
// kernel wrote are read. Output: bf16 out[r][d] (+ lse_out[r]), or, when
// `packed` is set, fp32 packed[r][0..D) with the lse at packed[r][D].
// Each part's weight e^(lse_s - M) is computed once into shared memory (in
// windows of kCombineWindow parts, rescaled as the running maximum grows).
constexpr int kCombineThreads = 128;
constexpr int kCombineWindow = 1024;

__device__ __forceinline__ float block_max(float v, float* red) {
  for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = red[0];
  for (int w = 1; w < kCombineThreads / 32; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  return m;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < kCombineThreads / 32; ++w) t += red[w];
  __syncthreads();
  return t;
}

// With kWait the CTA first waits (one thread, bounded) until every part's
// producer has published `wait`'s epoch; if that wait gives up it writes nothing.
template <bool kWait>
__global__ void __launch_bounds__(kCombineThreads)
    combine_kernel(const float* __restrict__ po, const float* __restrict__ pl, size_t o_row,
                   size_t o_part, size_t l_row, size_t l_part,
                   const int32_t* __restrict__ ctx_len, int Hq, int nparts, int pages_per_split,
                   int D, uint16_t* __restrict__ out, float* __restrict__ lse_out,
                   float* __restrict__ packed, PeerWait wait) {
  __shared__ float w[kCombineWindow];
  __shared__ float red[kCombineThreads / 32];
  pdl_wait();
  pdl_trigger();
  if constexpr (kWait) {
    __shared__ int ready;
    if (threadIdx.x == 0)
      ready = wait_epochs(wait.flags, wait.world, *wait.epoch_base + wait.epoch_add, wait.status);
    __syncthreads();
    if (!ready) return;
  }
  const int row = blockIdx.x;
  int ns = nparts;
  if (ctx_len != nullptr) {
    const int npages = (ctx_len[row / Hq] + kPage - 1) / kPage;
    ns = min(nparts, (npages + pages_per_split - 1) / pages_per_split);
  }
  const float* lse = pl + (size_t)row * l_row;
  const float* o = po + (size_t)row * o_row;
  constexpr int kDims = 4;  // dims per thread (D <= 512)
  // Up to kPrefetch parts: this thread's values are loaded into registers before the
  // weights are made, so those loads overlap the lse loads and the block reductions
  // (the sums take them in the same order as the general loop).
  constexpr int kPrefetch = 16;
  const bool prefetched = ns <= kPrefetch;
  float pv[kDims][kPrefetch];
  if (prefetched) {
#pragma unroll
    for (int j = 0; j < kDims; ++j) {
      const int d = threadIdx.x + j * kCombineThreads;
#pragma unroll
      for (int s = 0; s < kPrefetch; ++s)
        pv[j][s] = (s < ns && d < D) ? o[(size_t)s * o_part + d] : 0.f;
    }
  }
  float acc[kDims];
#pragma unroll
  for (int j = 0; j < kDims; ++j) acc[j] = 0.f;
  float M = -CUDART_INF_F, wsum = 0.f;
  for (int s0 = 0; s0 < ns; s0 += kCombineWindow) {
    const int n = min(kCombineWindow, ns - s0);
    float m = -CUDART_INF_F;
    for (int s = threadIdx.x; s < n; s += kCombineThreads) m = fmaxf(m, lse[(s0 + s) * l_part]);
    const float Mn = fmaxf(M, block_max(m, red));
    if (Mn == -CUDART_INF_F) continue;  // every part so far is empty
    float part = 0.f;
    for (int s = threadIdx.x; s < n; s += kCombineThreads) {
      const float ls = lse[(s0 + s) * l_part];
      const float e = ls == -CUDART_INF_F ? 0.f : __expf(ls - Mn);
      w[s] = e;
      part += e;
    }
    const float rescale = M == -CUDART_INF_F ? 0.f : __expf(M - Mn);
    wsum = wsum * rescale + block_sum(part, red);  // block_sum syncs: w[] is visible
    M = Mn;
#pragma unroll
    for (int j = 0; j < kDims; ++j) {
      const int d = threadIdx.x + j * kCombineThreads;
      if (d < D) {
        float a = acc[j] * rescale;
        if (prefetched) {  // one window: s0 = 0, n = ns
#pragma unroll
          for (int s = 0; s < kPrefetch; ++s)
            if (s < n) a = fmaf(w[s], pv[j][s], a);
        } else {
          for (int s = 0; s < n; ++s) a = fmaf(w[s], o[(size_t)(s0 + s) * o_part + d], a);
        }
        acc[j] = a;
      }
    }
    __syncthreads();  // w[] is rewritten by the next window
  }
  const bool empty = M == -CUDART_INF_F;
#pragma unroll
  for (int j = 0; j < kDims; ++j) {
    const int d = threadIdx.x + j * kCombineThreads;
    if (d < D) {
      const float val = empty ? 0.f : acc[j] / wsum;
      if (packed != nullptr)
        packed[(size_t)row * (D + 1) + d] = val;
      else
        out[(size_t)row * D + d] = f_to_bf16(val);
    }
  }
  if (threadIdx.x == 0) {
    const float l = empty ? -CUDART_INF_F : M + logf(wsum);
    if (packed != nullptr)
      packed[(size_t)row * (D + 1) + D] = l;
    else if (lse_out != nullptr)
      lse_out[row] = l;
  }
}

// The same merge for rows with many parts (a long sequence cut into many
// splits, or many devices): one CTA per (row, 32-dim tile), lane = dim, and
// the four warps take every fourth part, so each part's 128-byte slice is one
// coalesced load and the row's work spreads over D / 32 CTAs.
// With kPut the merged row is stored, packed, into every rank's receive slot
// for this rank (`put.dst`, over NVLink) instead of `packed`; the CTA that
// arrives last on `put.counter` resets it and publishes the epoch in every
// rank's flag for this rank (system-scope release).
template <bool kPut>
__global__ void __launch_bounds__(kCombineThreads)
    combine_tiled_kernel(const float* __restrict__ po, const float* __restrict__ pl,
                         size_t o_row, size_t o_part, size_t l_row, size_t l_part,
                         const int32_t* __restrict__ ctx_len, int Hq, int nparts,
                         int pages_per_split, int D, uint16_t* __restrict__ out,
                         float* __restrict__ lse_out, float* __restrict__ packed, PeerPut put) {
  __shared__ float w[kCombineWindow];
  __shared__ float red[kCombineThreads / 32];
  __shared__ float part_acc[kCombineThreads / 32][32];
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int d = blockIdx.y * 32 + lane;
  int ns = nparts;
  if (ctx_len != nullptr) {
    const int npages = (ctx_len[row / Hq] + kPage - 1) / kPage;
    ns = min(nparts, (npages + pages_per_split - 1) / pages_per_split);
  }
  const float* lse = pl + (size_t)row * l_row;
  const float* o = po + (size_t)row * o_row;
  constexpr int kStride = kCombineThreads / 32;
  // Up to kPrefetch parts per warp (kStride * kPrefetch parts in all), this lane's
  // values are loaded into registers before the weights are made, so the part loads
  // overlap the lse loads and the block reductions; the sums below take them in the
  // same order as the loads of the general loop.
  constexpr int kPrefetch = 32;
  const bool prefetched = ns <= kStride * kPrefetch;
  const int cnt_w = ns > warp ? (ns - warp + kStride - 1) / kStride : 0;  // parts of this warp
  float pv[kPrefetch];
  if (prefetched) {
#pragma unroll
    for (int i = 0; i < kPrefetch; ++i)
      pv[i] = (i < cnt_w && d < D) ? o[(size_t)(warp + kStride * i) * o_part + d] : 0.f;
  }
  float acc = 0.f, M = -CUDART_INF_F, wsum = 0.f;
  for (int s0 = 0; s0 < ns; s0 += kCombineWindow) {
    const int n = min(kCombineWindow, ns - s0);
    float m = -CUDART_INF_F;
    for (int s = threadIdx.x; s < n; s += kCombineThreads) m = fmaxf(m, lse[(s0 + s) * l_part]);
    const float Mn = fmaxf(M, block_max(m, red));
    if (Mn == -CUDART_INF_F) continue;
    float part = 0.f;
    for (int s = threadIdx.x; s < n; s += kCombineThreads) {
      const float ls = lse[(s0 + s) * l_part];
      const float e = ls == -CUDART_INF_F ? 0.f : __expf(ls - Mn);
      w[s] = e;
      part += e;
    }
    const float rescale = M == -CUDART_INF_F ? 0.f : __expf(M - Mn);
    wsum = wsum * rescale + block_sum(part, red);
    M = Mn;
    float a = acc * rescale;
    if (d < D && prefetched) {  // one window: s0 = 0, n = ns
      float a1 = 0.f, a2 = 0.f, a3 = 0.f;
      int done = 0;
#pragma unroll
      for (int i = 0; i < kPrefetch; i += 4) {
        if (i + 3 < cnt_w) {
          a = fmaf(w[warp + kStride * i], pv[i], a);
          a1 = fmaf(w[warp + kStride * (i + 1)], pv[i + 1], a1);
          a2 = fmaf(w[warp + kStride * (i + 2)], pv[i + 2], a2);
          a3 = fmaf(w[warp + kStride * (i + 3)], pv[i + 3], a3);
          done = i + 4;
        }
      }
#pragma unroll
      for (int i = 0; i < kPrefetch; ++i)
        if (i >= done && i < cnt_w) a = fmaf(w[warp + kStride * i], pv[i], a);
      a += (a1 + a2) + a3;
    } else if (d < D) {
      // Four parts in flight per warp: the loads do not wait on the sum chain.
      float a1 = 0.f, a2 = 0.f, a3 = 0.f;
      int s = warp;
      for (; s + 3 * kStride < n; s += 4 * kStride) {
        const float v0 = o[(size_t)(s0 + s) * o_part + d];
        const float v1 = o[(size_t)(s0 + s + kStride) * o_part + d];
        const float v2 = o[(size_t)(s0 + s + 2 * kStride) * o_part + d];
        const float v3 = o[(size_t)(s0 + s + 3 * kStride) * o_part + d];
        a = fmaf(w[s], v0, a);
        a1 = fmaf(w[s + kStride], v1, a1);
        a2 = fmaf(w[s + 2 * kStride], v2, a2);
        a3 = fmaf(w[s + 3 * kStride], v3, a3);
      }
      for (; s < n; s += kStride) a = fmaf(w[s], o[(size_t)(s0 + s) * o_part + d], a);
      a += (a1 + a2) + a3;
    }
    acc = a;
    __syncthreads();
  }
  part_acc[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && d < D) {
    float total = 0.f;
#pragma unroll
    for (int k = 0; k < kCombineThreads / 32; ++k) total += part_acc[k][lane];
    const bool empty = M == -CUDART_INF_F;
    const float val = empty ? 0.f : total / wsum;
    const float l = empty ? -CUDART_INF_F : M + logf(wsum);
    if constexpr (kPut) {
      put.local[(size_t)row * (D + 1) + d] = val;
      if (blockIdx.y == 0 && lane == 0) put.local[(size_t)row * (D + 1) + D] = l;
    } else {
      if (packed != nullptr)
        packed[(size_t)row * (D + 1) + d] = val;
      else
        out[(size_t)row * D + d] = f_to_bf16(val);
      if (blockIdx.y == 0 && lane == 0) {
        if (packed != nullptr)
          packed[(size_t)row * (D + 1) + D] = l;
        else if (lse_out != nullptr)
          lse_out[row] = l;
      }
    }
  }
  if constexpr (kPut) {
    // The CTA that arrives last copies the whole packed block to every rank
    // and publishes the epoch: one system-scope fence per launch.
    __shared__ int last;
    __syncthreads();  // this CTA's rows precede thread 0's fence and arrival
    if (threadIdx.x == 0) {
      __threadfence();
      last = atomicAdd(put.counter, 1u) == gridDim.x * gridDim.y - 1;
      if (last) __threadfence();  // every other CTA's rows are visible from here
    }
    __syncthreads();
    if (last) {
      const uint4* src = reinterpret_cast<const uint4*>(put.local);
      const int chunks = (int)(gridDim.x * (size_t)(D + 1) * 4 / 16);
      for (int p = 0; p < put.world; ++p) {
        uint4* dst = reinterpret_cast<uint4*>(put.dst[p]);
        for (int i = threadIdx.x; i < chunks; i += blockDim.x) dst[i] = src[i];
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        *put.counter = 0;  // ready for the next launch (stream order)
        __threadfence_system();
        const unsigned int epoch = *put.epoch_base + put.epoch_add;
        for (int p = 0; p < put.world; ++p) st_release_sys(put.flag[p], epoch);
      }
    }
  }
}

}  // namespace

// Launches the merge of `rows` rows of `nparts` parts: per-row CTAs for few
// parts, (row, dim-tile) CTAs for many.
void launch_combine(const float* po, const float* pl, size_t o_row, size_t o_part, size_t l_row,
                    size_t l_part, const int32_t* ctx_len, int Hq, int nparts,
                    int pages_per_split, int D, int rows, uint16_t* out, float* lse_out,
                    float* packed, cudaStream_t s) {
  if (nparts >= 16) {
    dim3 grid(rows, (D + 31) / 32);
    launch_pdl(combine_tiled_kernel<false>, grid, dim3(kCombineThreads), 0, s, po, pl, o_row,
               o_part, l_row, l_part, ctx_len, Hq, nparts, pages_per_split, D, out, lse_out,
               packed, PeerPut{});
  } else {
    launch_pdl(combine_kernel<false>, dim3(rows), dim3(kCombineThreads), 0, s, po, pl, o_row,
               o_part, l_row, l_part, ctx_len, Hq, nparts, pages_per_split, D, out, lse_out,
               packed, PeerWait{});
  }
}

namespace {

// Launch shape: warps per CTA and shared-memory stages (one page each) per warp.
#ifndef SC_ATTN_WARPS
#define SC_ATTN_WARPS 4
#endif
#ifndef SC_ATTN_STAGES
#define SC_ATTN_STAGES 3
#endif
constexpr int kWarpsPerCta = SC_ATTN_WARPS;
constexpr int kStages = SC_ATTN_STAGES;

template <int D>
int launch_decode(const uint16_t* q, const uint16_t* kv_pool, const int32_t* block_table,
                  const int32_t* ctx_len, const int32_t* seq_order, int B, int Hq, int Hkv,
                  int max_pages,
                  int pages_per_split, int num_splits, float scale, float* part_out,
                  float* part_lse, uint16_t* out, float* lse_out, float* packed,
                  long long num_pages, const PeerPut* put, const FusedArgs* fused,
                  cudaStream_t s) {
  using S = AttnShape<D>;
  constexpr int NW = kWarpsPerCta, NST = kStages;
  const size_t smem = (size_t)NW * NST * S::STAGE_BYTES + NW * NST * sizeof(uint64_t);
  auto kernel = fused != nullptr ? paged_decode_kernel<D, NW, NST, true>
                                 : paged_decode_kernel<D, NW, NST, false>;
  static int configured[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[fused != nullptr][dev]) {
    cudaError_t err =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess)
      return set_error(SC_ERR_CUDA, "sc_paged_decode_attention: smem attribute: %s",
                       cudaGetErrorString(err));
    configured[fused != nullptr][dev] = 1;
  }
  const int G = Hq / Hkv;
  const int HG = (G + kHeadsPerTile - 1) / kHeadsPerTile;
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid(num_splits, Hkv * HG, B);
  cudaError_t err = launch_pdl(kernel, grid, dim3(NW * 32), smem, s, q, kv_pool, block_table,
                               ctx_len, seq_order, Hq, Hkv, G, HG, max_pages, pages_per_split,
                               num_splits, scale_log2, part_out, part_lse, out, lse_out, packed,
                               num_pages, device_status_word(),
                               fused != nullptr ? *fused : FusedArgs{});
  if (err != cudaSuccess)
    return set_error(SC_ERR_CUDA, "sc_paged_decode_attention: launch: %s",
                     cudaGetErrorString(err));
  if (int rc = check_launch("sc_paged_decode_attention")) return rc;
  if (fused != nullptr && fused->merge) return SC_OK;  // the splits merged themselves
  if (put != nullptr) {  // the entry guarantees num_splits > 1
    dim3 cgrid(B * Hq, (D + 31) / 32);
    launch_pdl(combine_tiled_kernel<true>, cgrid, dim3(kCombineThreads), 0, s,
               (const float*)part_out, (const float*)part_lse, (size_t)num_splits * D, (size_t)D,
               (size_t)num_splits, (size_t)1, ctx_len, Hq, num_splits, pages_per_split, D,
               (uint16_t*)nullptr, (float*)nullptr, (float*)nullptr, *put);
    return check_launch("sc_paged_decode_attention_exchange(combine)");
  }
  if (num_splits > 1) {
    launch_combine(part_out, part_lse, (size_t)num_splits * D, D, num_splits, 1, ctx_len, Hq,
                   num_splits, pages_per_split, D, B * Hq, out, lse_out, packed, s);
    return check_launch("sc_paged_decode_attention(combine)");
  }
  return SC_OK;
}

}  // namespace
}  // namespace sc

namespace sc {
namespace {
int decode_entry(const char* name, const sc_bf16* q, const sc_bf16* kv_pool, int64_t num_pages,
                 const int32_t* block_table, const int32_t* ctx_len, const int32_t* seq_order,
                 int B, int Hq, int Hkv,
                 int D, int P, int max_pages, int pages_per_split, int num_splits, float scale,
                 float* part_out, float* part_lse, sc_bf16* out, float* lse_out, float* packed,
                 const PeerPut* put, void* stream, const FusedArgs* fused = nullptr) {
  SC_REQUIRE(q && kv_pool && block_table && ctx_len && (out || packed || put), SC_ERR_INVALID,
             "%s: null pointer", name);
  SC_REQUIRE(B >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0, SC_ERR_INVALID,
             "%s: bad heads Hq=%d Hkv=%d", name, Hq, Hkv);
  SC_REQUIRE(P == sc::kPage, SC_ERR_UNSUPPORTED, "%s: page size %d != 16", name, P);
  SC_REQUIRE(max_pages > 0 && pages_per_split > 0 && num_splits > 0, SC_ERR_INVALID,
             "%s: bad split plan max_pages=%d pages_per_split=%d num_splits=%d", name, max_pages,
             pages_per_split, num_splits);
  SC_REQUIRE(num_splits == 1 || (part_out && part_lse), SC_ERR_INVALID,
             "%s: num_splits > 1 needs part_out and part_lse", name);
  SC_REQUIRE(num_splits <= 65535 && B <= 65535 && Hkv * ((Hq / Hkv + 7) / 8) <= 65535,
             SC_ERR_INVALID, "%s: grid too large", name);
  SC_REQUIRE(num_pages > 0, SC_ERR_INVALID, "%s: num_pages=%lld", name, (long long)num_pages);
  if (B == 0) return SC_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (D) {
    case 64:
      return launch_decode<64>(q, kv_pool, block_table, ctx_len, seq_order, B, Hq, Hkv,
                                 max_pages,
                                   pages_per_split, num_splits, scale, part_out, part_lse, out,
                                   lse_out, packed, num_pages, put, fused, s);
    case 128:
      return launch_decode<128>(q, kv_pool, block_table, ctx_len, seq_order, B, Hq, Hkv,
                                 max_pages,
                                    pages_per_split, num_splits, scale, part_out, part_lse, out,
                                    lse_out, packed, num_pages, put, fused, s);
    case 256:
      return launch_decode<256>(q, kv_pool, block_table, ctx_len, seq_order, B, Hq, Hkv,
                                 max_pages,
                                    pages_per_split, num_splits, scale, part_out, part_lse, out,
                                    lse_out, packed, num_pages, put, fused, s);
    default:
      return set_error(SC_ERR_UNSUPPORTED, "%s: D=%d not in {64,128,256}", name, D);
  }
}
}  // namespace
}  // namespace sc

extern "C" int sc_paged_decode_attention(const sc_bf16* q, const sc_bf16* kv_pool,
                                         int64_t num_pages, const int32_t* block_table,
                                         const int32_t* ctx_len, const int32_t* seq_order, int B,
                                         int Hq, int Hkv, int D,
                                         int P, int max_pages, int pages_per_split,
                                         int num_splits, float scale,
                                         float* part_out, float* part_lse, sc_bf16* out,
                                         float* lse_out, void* stream) {
  SC_REQUIRE(out != nullptr, SC_ERR_INVALID, "sc_paged_decode_attention: null pointer");
  return sc::decode_entry("sc_paged_decode_attention", q, kv_pool, num_pages, block_table,
                          ctx_len, seq_order, B, Hq, Hkv, D, P, max_pages, pages_per_split,
                          num_splits,
                          scale, part_out, part_lse, out, lse_out, nullptr, nullptr, stream);
}

extern "C" int sc_paged_decode_attention_fused(
    const sc_bf16* q, const sc_bf16* k_new, const sc_bf16* v_new, const int64_t* slot_mapping,
    sc_bf16* kv_pool, int64_t num_pages, const int32_t* block_table, const int32_t* ctx_len,
    const int32_t* seq_order, int B, int Hq, int Hkv, int D, int P, int max_pages,
    int pages_per_split, int num_splits, float scale, float* part_out, float* part_lse,
    unsigned int* counters, sc_bf16* out, float* lse_out, float* packed, int in_kernel_merge,
    void* stream) {
  const char* name = "sc_paged_decode_attention_fused";
  SC_REQUIRE(k_new && v_new && slot_mapping, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE((out != nullptr) != (packed != nullptr), SC_ERR_INVALID,
             "%s: give exactly one of out and packed", name);
  const bool merge = in_kernel_merge && num_splits > 1 && num_splits <= sc::kFusedMergeParts;
  SC_REQUIRE(!merge || counters != nullptr, SC_ERR_INVALID,
             "%s: the in-kernel merge needs the arrival counters", name);
  SC_REQUIRE(((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 15) ==
                 0 && (reinterpret_cast<uintptr_t>(out) & 7) == 0,
             SC_ERR_INVALID, "%s: k_new and v_new must be 16-byte aligned, out 8-byte aligned",
             name);
  sc::FusedArgs fa;
  fa.k_new = reinterpret_cast<const uint16_t*>(k_new);
  fa.v_new = reinterpret_cast<const uint16_t*>(v_new);
  fa.slot_mapping = slot_mapping;
  fa.pool = reinterpret_cast<uint16_t*>(kv_pool);
  fa.counters = counters;
  fa.merge = merge ? 1 : 0;
  return sc::decode_entry(name, q, kv_pool, num_pages, block_table, ctx_len, seq_order, B, Hq,
                          Hkv, D, P, max_pages, pages_per_split, num_splits, scale, part_out,
                          part_lse, out, lse_out, packed, nullptr, stream, &fa);
}

extern "C" int sc_paged_decode_attention_packed(const sc_bf16* q, const sc_bf16* kv_pool,
                                                int64_t num_pages, const int32_t* block_table,
                                                const int32_t* ctx_len, int B, int Hq, int Hkv,
                                                int D, int P, int max_pages,
                                                int pages_per_split, int num_splits, float scale,
                                                float* part_out, float* part_lse, float* packed,
                                                void* stream) {
  SC_REQUIRE(packed != nullptr, SC_ERR_INVALID, "sc_paged_decode_attention_packed: null pointer");
  return sc::decode_entry("sc_paged_decode_attention_packed", q, kv_pool, num_pages,
                          block_table, ctx_len, nullptr, B, Hq, Hkv, D, P, max_pages,
                          pages_per_split,
                          num_splits, scale, part_out, part_lse, nullptr, nullptr, packed,
                          nullptr, stream);
}

extern "C" int sc_attention_combine_packed(const float* gathered, int nparts, int rows, int D,
                                           sc_bf16* out, float* lse_out, void* stream) {
  const char* name = "sc_attention_combine_packed";
  SC_REQUIRE(gathered && out, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(rows >= 0 && nparts > 0 && D > 0 && D <= 512, SC_ERR_INVALID,
             "%s: rows=%d nparts=%d D=%d (D <= 512)", name, rows, nparts, D);
  if (rows == 0) return SC_OK;
  const size_t stride = (size_t)D + 1;
  sc::launch_combine(gathered, gathered + D, stride, (size_t)rows * stride, stride,
                     (size_t)rows * stride, nullptr, 1, nparts, 1, D, rows, out, lse_out, nullptr,
                     static_cast<cudaStream_t>(stream));
  return sc::check_launch(name);
}

extern "C" int sc_paged_decode_attention_exchange(
    const sc_bf16* q, const sc_bf16* kv_pool, int64_t num_pages, const int32_t* block_table,
    const int32_t* ctx_len, int B, int Hq, int Hkv, int D, int P, int max_pages,
    int pages_per_split, int num_splits, float scale, float* part_out, float* part_lse,
    float* packed, float* const* peer_dst, unsigned int* const* peer_flag,
    unsigned int* counter, const unsigned int* epoch_base, unsigned int epoch_add, int world,
    void* stream) {
  const char* name = "sc_paged_decode_attention_exchange";
  SC_REQUIRE(packed && peer_dst && peer_flag && counter && epoch_base, SC_ERR_INVALID,
             "%s: null pointer", name);
  SC_REQUIRE((reinterpret_cast<uintptr_t>(packed) & 15) == 0 &&
                 ((long long)B * Hq * (D + 1) * 4) % 16 == 0,
             SC_ERR_INVALID, "%s: packed must be 16-byte aligned and B*Hq*(D+1)*4 a multiple "
             "of 16", name);
  SC_REQUIRE(world > 0 && world <= 1024, SC_ERR_INVALID, "%s: world=%d", name, world);
  SC_REQUIRE(num_splits > 1 && B > 0, SC_ERR_INVALID,
             "%s: needs num_splits > 1 (got %d) and B > 0 (got %d)", name, num_splits, B);
  SC_REQUIRE((long long)B * Hq <= 65535, SC_ERR_INVALID, "%s: B*Hq=%lld rows", name,
             (long long)B * Hq);
  sc::PeerPut put;
  put.local = packed;
  put.dst = peer_dst;
  put.flag = peer_flag;
  put.counter = counter;
  put.epoch_base = epoch_base;
  put.epoch_add = epoch_add;
  put.world = world;
  return sc::decode_entry(name, q, kv_pool, num_pages, block_table, ctx_len, nullptr, B, Hq, Hkv,
                          D, P, max_pages, pages_per_split, num_splits, scale, part_out, part_lse,
                          nullptr, nullptr, nullptr, &put, stream);
}

extern "C" int sc_attention_combine_exchange(const float* gathered, const unsigned int* flags,
                                             const unsigned int* epoch_base,
                                             unsigned int epoch_add, int nparts, int rows, int D,
                                             sc_bf16* out, float* lse_out, void* stream) {
  const char* name = "sc_attention_combine_exchange";
  SC_REQUIRE(gathered && flags && epoch_base && out, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(rows >= 0 && nparts > 0 && nparts <= 1024 && D > 0 && D <= 512, SC_ERR_INVALID,
             "%s: rows=%d nparts=%d D=%d (D <= 512)", name, rows, nparts, D);
  if (rows == 0) return SC_OK;
  const size_t stride = (size_t)D + 1;
  sc::PeerWait wait;
  wait.flags = flags;
  wait.epoch_base = epoch_base;
  wait.epoch_add = epoch_add;
  wait.world = nparts;
  wait.status = sc::device_status_word();
  sc::launch_pdl(sc::combine_kernel<true>, dim3(rows), dim3(sc::kCombineThreads), 0,
                 static_cast<cudaStream_t>(stream), gathered, (const float*)(gathered + D),
                 stride, (size_t)rows * stride, stride, (size_t)rows * stride,
                 (const int32_t*)nullptr, 1, nparts, 1, D, reinterpret_cast<uint16_t*>(out),
                 lse_out, (float*)nullptr, wait);
  return sc::check_launch(name);
}

extern "C" int sc_attention_combine(const float* part_out, const float* part_lse, int rows,
                                    int nparts, int D, sc_bf16* out, float* lse_out,
                                    void* stream) {
  const char* name = "sc_attention_combine";
  SC_REQUIRE(part_out && part_lse && out, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(rows >= 0 && nparts > 0 && D > 0 && D <= 512, SC_ERR_INVALID,
             "%s: rows=%d nparts=%d D=%d (D <= 512)", name, rows, nparts, D);
  if (rows == 0) return SC_OK;
  sc::launch_combine(part_out, part_lse, (size_t)nparts * D, D, nparts, 1, nullptr, 1, nparts, 1,
                     D, rows, out, lse_out, nullptr, static_cast<cudaStream_t>(stream));
  return sc::check_launch(name);
}

// ---------------------------------------------------------------------------
// Split-K decode attention for callers that cannot allocate device memory.
//
// The split partials live in one file-scope device array instead of caller
// scratch. Every GPU that loads this library holds the array (32 MiB) until
// the process exits. Host code must not pass the array's name to a kernel:
// on the host that name is only a stand-in symbol, so the device address is
// looked up once per device with cudaGetSymbolAddress and cached.
namespace sc {
namespace {

__device__ __align__(256) float g_noalloc_partials[SC_NOALLOC_SCRATCH_FLOATS];

std::mutex g_noalloc_mutex;
float* g_noalloc_addr[64] = {};

// Device address of g_noalloc_partials on the current device (set-up on the
// first call per device), or nullptr with the error recorded.
float* noalloc_scratch(const char* name) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess || dev < 0 || dev >= 64) {
    set_error(SC_ERR_CUDA, "%s: no current device (%s)", name, cudaGetErrorString(err));
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (err != cudaSuccess || p == nullptr) {
      set_error(SC_ERR_CUDA, "%s: cudaGetSymbolAddress failed: %s", name,
                cudaGetErrorString(err));
      return nullptr;
    }
    g_noalloc_addr[dev] = static_cast<float*>(p);
  }
  return g_noalloc_addr[dev];
}

}  // namespace
}  // namespace sc

extern "C" int sc_paged_decode_attention_noalloc(const sc_bf16* q, const sc_bf16* kv_pool,
                                                 int64_t num_pages, const int32_t* block_table,
                                                 const int32_t* ctx_len, int B, int Hq, int Hkv,
                                                 int D, int P, int max_pages, int pages_per_split,
                                                 int num_splits, float scale, sc_bf16* out,
                                                 float* lse_out, void* stream) {
  const char* name = "sc_paged_decode_attention_noalloc";
  SC_REQUIRE(B >= 0 && Hq > 0 && num_splits > 0 && D > 0, SC_ERR_INVALID,
             "%s: bad sizes B=%d Hq=%d num_splits=%d D=%d", name, B, Hq, num_splits, D);
  // Partials [B, Hq, num_splits, D] followed by their lse [B, Hq, num_splits].
  const long long rows = (long long)B * Hq * num_splits;
  const long long need = rows * (D + 1LL);
  SC_REQUIRE(num_splits == 1 || need <= SC_NOALLOC_SCRATCH_FLOATS, SC_ERR_INVALID,
             "%s: B*Hq*num_splits*(D+1) = %lld floats exceeds the built-in scratch of %d floats "
             "(32 MiB); use fewer splits (larger pages_per_split) or sc_paged_decode_attention "
             "with caller scratch",
             name, need, SC_NOALLOC_SCRATCH_FLOATS);
  float* part_out = nullptr;
  float* part_lse = nullptr;
  if (num_splits > 1) {  // one split writes the output directly and needs no scratch
    float* scratch = sc::noalloc_scratch(name);
    if (scratch == nullptr) return SC_ERR_CUDA;
    part_out = scratch;
    part_lse = scratch + rows * D;
  }
  return sc_paged_decode_attention(q, kv_pool, num_pages, block_table, ctx_len, nullptr, B, Hq,
                                   Hkv, D, P,
                                   max_pages, pages_per_split, num_splits, scale, part_out,
                                   part_lse, out, lse_out, stream);
}
