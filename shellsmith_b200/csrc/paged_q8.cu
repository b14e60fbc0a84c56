// 8-bit KV pages: affine quantisation in groups of 64 on append, and split-K
// decode attention that feeds the codes to the tensor cores directly.
//
// Reference: the cache_precision="8bit" request option
// (studio_compute/inference.py:87-94), which turns each layer's cache into an
// mlx-vlm QuantizedKVCache: every K and V row quantised along D in groups of
// 64 with 8 bits, a scale and a bias per group (w = scale * code + bias), and
// attention computed on the dequantised rows. The library's exact rounding of
// scale and bias is not in the reference tree; this build's rule is
//   scale = bf16((max - min) / 255), bias = bf16(min),
//   code  = clamp(rint((w - bias) / scale), 0, 255)   (0 when scale == 0),
// all fp32 IEEE arithmetic, restated bit for bit by oracle.attention.quantize_q8.
//
// Page block (one page, one kv head), D in {128, 256}, G = D / 64:
//   K codes  [16 tokens][D]: row t, 32-bit word pw = (w + 4 (t & 7)) mod D/4,
//            where word w = 4 kk + c holds dims 16 kk + {2c, 2c+1, 2c+8, 2c+9}
//            (the bytes an m16n8k16 A fragment takes from row t, rotated per
//            row so the warp's loads hit 32 distinct banks)
//   V codes  V^T [D dims][16 tokens]: row d, word c holds tokens
//            {2c, 2c+1, 2c+8, 2c+9} (the A fragment of O^T = V^T P^T)
//   K scale, K bias, V scale, V bias: [16 tokens][G] bf16 each
// 8704 bytes for D = 256 against 16384 for a bf16 page: attention reads half.
//
// Attention. A code byte n becomes the fp16 value 1024 + n with one byte
// permute (0x64 high byte), so K and V^T fragments go to mma.m16n8k16 in fp16
// without a dequantise pass. Scale and bias are applied per (token, group):
//   score(t) = sum_g ks[t][g] * (sum_{d in g} (1024 + n[t][d]) q[d])
//              + sum_g (kb[t][g] - 1024 ks[t][g]) * qsum_g
//   O[d]     = sum_t (p[t] vs[t][g]) (1024 + n[t][d])
//              + sum_t (p[t] vb[t][g] - 1024 fp16(p[t] vs[t][g]))
// with qsum_g the sum of the (fp16) query over group g. The score MMA keeps
// one accumulator per group; the probabilities are scaled per group into the
// B operand of the value MMA; the last term is a per-(group, head) sum that
// each lane carries (rescaled with the running max) and the warp reduces once.
// Everything else (splits, online softmax, warp merge, combine) is the bf16
// kernel's.
#include <cuda_fp16.h>
#include <math_constants.h>

#include "attention_internal.cuh"
#include "common.cuh"

namespace sc {
namespace {

constexpr int kPage = 16;
constexpr int kGroup = 64;
constexpr int kHeadsPerTile = 8;

template <int D>
struct Q8 {
  static constexpr int G = D / kGroup;
  static constexpr int WORDS = D / 4;
  static constexpr int KSTEPS = D / 16;
  static constexpr int K_BYTES = kPage * D;
  static constexpr int V_BYTES = kPage * D;
  static constexpr int SB_BYTES = kPage * G * 2;
  static constexpr int OFF_V = K_BYTES;
  static constexpr int OFF_KS = K_BYTES + V_BYTES;
  static constexpr int OFF_KB = OFF_KS + SB_BYTES;
  static constexpr int OFF_VS = OFF_KB + SB_BYTES;
  static constexpr int OFF_VB = OFF_VS + SB_BYTES;
  static constexpr int BLOCK = OFF_VB + SB_BYTES;
};

__host__ __device__ inline int q8_block_bytes(int D) {
  return 2 * kPage * D + 4 * kPage * (D / kGroup) * 2;
}

// Byte of K code (token t, dim d) and of V code (token t, dim d) in a page block.
__device__ __forceinline__ int k_code_byte(int D, int t, int d) {
  const int kk = d >> 4, r = d & 15;
  const int c = (r & 7) >> 1, byte = (r & 1) + ((r >> 3) << 1);
  const int pw = (4 * kk + c + 4 * (t & 7)) & (D / 4 - 1);
  return t * D + pw * 4 + byte;
}
__device__ __forceinline__ int v_code_byte(int D, int t, int d) {
  const int c = (t & 7) >> 1, byte = (t & 1) + ((t >> 3) << 1);
  return kPage * D + d * 16 + c * 4 + byte;
}

__device__ __forceinline__ float bfr(float x) { return bf16_to_f(f_to_bf16(x)); }

// One warp per (token, kv head, K or V): lanes hold D/32 consecutive values;
// a group of 64 spans 64 / (D/32) lanes.
template <int D>
__global__ void __launch_bounds__(256)
    kv_append_q8_kernel(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                        uint8_t* __restrict__ pool, const int64_t* __restrict__ slot_mapping,
                        int ntok, int Hkv, long long num_pages, unsigned int* status) {
  using S = Q8<D>;
  constexpr int VPL = D / 32, LPG = kGroup / VPL;
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (long long)ntok * Hkv * 2) return;
  const int which = (int)(wid & 1);  // 0: K, 1: V
  const long long th = wid >> 1;
  const int tok = (int)(th / Hkv), h = (int)(th - (long long)tok * Hkv);
  const int64_t slot = slot_mapping[tok];
  if (slot < 0) return;
  const long long page = slot / kPage;
  const int t = (int)(slot - page * kPage);
  if (page >= num_pages) {
    if (lane == 0) flag_device(status, DEV_BAD_INDEX);
    return;
  }
  const uint16_t* src = (which ? v : k) + ((size_t)tok * Hkv + h) * D + lane * VPL;
  float x[VPL];
#pragma unroll
  for (int e = 0; e < VPL; ++e) x[e] = bf16_to_f(src[e]);
  float mn = x[0], mx = x[0];
#pragma unroll
  for (int e = 1; e < VPL; ++e) {
    mn = fminf(mn, x[e]);
    mx = fmaxf(mx, x[e]);
  }
#pragma unroll
  for (int off = 1; off < LPG; off <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  }
  const float scale = bfr(__fdiv_rn(__fsub_rn(mx, mn), 255.f));
  const float bias = bfr(mn);
  uint8_t* blk = pool + ((size_t)page * Hkv + h) * S::BLOCK;
#pragma unroll
  for (int e = 0; e < VPL; ++e) {
    const int d = lane * VPL + e;
    float code = 0.f;
    if (scale > 0.f)
      code = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(x[e], bias), scale)), 0.f), 255.f);
    blk[which ? v_code_byte(D, t, d) : k_code_byte(D, t, d)] = (uint8_t)code;
  }
  if (lane % LPG == 0) {
    const int g = lane / LPG;
    uint16_t* sb = reinterpret_cast<uint16_t*>(blk + (which ? S::OFF_VS : S::OFF_KS));
    sb[t * S::G + g] = f_to_bf16(scale);
    sb[S::SB_BYTES / 2 + t * S::G + g] = f_to_bf16(bias);
  }
}

// Reads tokens back in plain order: codes [ntok][Hkv][2][D] u8, scale/bias
// [ntok][Hkv][2][G][2] bf16 (for tests and debugging).
template <int D>
__global__ void kv_gather_q8_kernel(const uint8_t* __restrict__ pool,
                                    const int64_t* __restrict__ slot_mapping, int ntok, int Hkv,
                                    long long num_pages, uint8_t* __restrict__ codes,
                                    uint16_t* __restrict__ sb, unsigned int* status) {
  using S = Q8<D>;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)ntok * Hkv * 2 * D) return;
  const int d = (int)(idx % D);
  const long long r = idx / D;  // (tok, h, which)
  const int which = (int)(r & 1);
  const int h = (int)((r >> 1) % Hkv);
  const int tok = (int)((r >> 1) / Hkv);
  const int64_t slot = slot_mapping[tok];
  const bool live = slot >= 0 && slot / kPage < num_pages;
  if (slot >= 0 && !live && d == 0) flag_device(status, DEV_BAD_INDEX);
  const long long page = live ? slot / kPage : 0;
  const int t = live ? (int)(slot % kPage) : 0;
  const uint8_t* blk = pool + ((size_t)page * Hkv + h) * S::BLOCK;
  codes[idx] = live ? blk[which ? v_code_byte(D, t, d) : k_code_byte(D, t, d)] : 0;
  if (d < 2 * S::G) {
    const int g = d >> 1, part = d & 1;  // part 0: scale, 1: bias
    const uint16_t* src =
        reinterpret_cast<const uint16_t*>(blk + (which ? S::OFF_VS : S::OFF_KS));
    sb[r * 2 * S::G + 2 * g + part] = live ? src[part * (S::SB_BYTES / 2) + t * S::G + g] : 0;
  }
}

__device__ __forceinline__ void mma_f16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_f16x2(uint32_t x) {
  return __half22float2(*reinterpret_cast<const __half2*>(&x));
}
// Codes of bytes 0, 1 (lo) or 2, 3 (hi) of w as a pair of fp16 values 1024 + code.
__device__ __forceinline__ uint32_t codes_lo(uint32_t w) {
  return __byte_perm(w, 0x64646464u, 0x4140);
}
__device__ __forceinline__ uint32_t codes_hi(uint32_t w) {
  return __byte_perm(w, 0x64646464u, 0x4342);
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
// N (2 or 4) bf16 values of shared memory, 2N-byte aligned, as floats.
template <int N>
__device__ __forceinline__ void lds_bf16(uint32_t addr, float* out) {
  static_assert(N == 2 || N == 4, "two or four values");
  if constexpr (N == 4) {
    uint32_t a, b;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr));
    out[0] = bf16_lo(a);
    out[1] = bf16_hi(a);
    out[2] = bf16_lo(b);
    out[3] = bf16_hi(b);
  } else {
    const uint32_t a = lds32(addr);
    out[0] = bf16_lo(a);
    out[1] = bf16_hi(a);
  }
}

template <int D, int NW, int NSTAGE>
__global__ void __launch_bounds__(NW * 32)
    paged_decode_q8_kernel(const uint16_t* __restrict__ q, const uint8_t* __restrict__ pool,
                           const int32_t* __restrict__ block_table,
                           const int32_t* __restrict__ ctx_len,
                           const int32_t* __restrict__ seq_order, int Hq, int Hkv, int G, int HG,
                           int max_pages, int pages_per_split, int num_splits, float scale_log2,
                           float* __restrict__ part_out, float* __restrict__ part_lse,
                           uint16_t* __restrict__ out, float* __restrict__ lse_out,
                           long long num_pages, unsigned int* status) {
  using S = Q8<D>;
  constexpr int NG = S::G;
  constexpr int KK_PER_G = kGroup / 16;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NW * NSTAGE * S::BLOCK);
  if (status != nullptr && (*reinterpret_cast<volatile unsigned int*>(status) & DEV_WAIT_TIMEOUT))
    return;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y / HG;
  const int hg = blockIdx.y - kvh * HG;
  const int b = seq_order != nullptr ? seq_order[blockIdx.z] : (int)blockIdx.z;
  if (b < 0 || b >= (int)gridDim.z) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) flag_device(status, DEV_BAD_INDEX);
    return;
  }
  const int L = checked_ctx_len(ctx_len[b], kPage, max_pages, pages_per_split, num_splits,
                                status, split == 0 && blockIdx.y == 0 && threadIdx.x == 0);
  const int npages = (L + kPage - 1) / kPage;
  const int p_begin = split * pages_per_split;
  if (npages == 0 && split == 0) {  // nothing to attend: zero output, lse = -inf
    for (int idx = threadIdx.x; idx < min(kHeadsPerTile, G - hg * kHeadsPerTile) * D;
         idx += blockDim.x) {
      const size_t row = (size_t)b * Hq + kvh * G + hg * kHeadsPerTile + idx / D;
      if (num_splits == 1) {
        out[row * D + idx % D] = 0;
        if (idx % D == 0 && lse_out != nullptr) lse_out[row] = -CUDART_INF_F;
      }
    }
    return;
  }
  if (p_begin >= npages) return;
  const int n_here = min(npages, p_begin + pages_per_split) - p_begin;
  const int heads_here = min(kHeadsPerTile, G - hg * kHeadsPerTile);
  const int head0 = kvh * G + hg * kHeadsPerTile;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g8 = lane >> 2, c4 = lane & 3;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NW * NSTAGE; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // Q^T as the fp16 B operand (head g8), and the per-group query sums of this
  // lane's accumulator heads 2c, 2c+1.
  uint32_t qf[S::KSTEPS][2];
  float qsum[NG][2];
  {
    const bool valid = g8 < heads_here;
    const uint16_t* qp = q + ((size_t)b * Hq + head0 + (valid ? g8 : 0)) * D;
    float part[NG];
#pragma unroll
    for (int gr = 0; gr < NG; ++gr) part[gr] = 0.f;
#pragma unroll
    for (int kk = 0; kk < S::KSTEPS; ++kk) {
      const uint32_t lo = valid ? *reinterpret_cast<const uint32_t*>(qp + 16 * kk + 2 * c4) : 0u;
      const uint32_t hi =
          valid ? *reinterpret_cast<const uint32_t*>(qp + 16 * kk + 8 + 2 * c4) : 0u;
      qf[kk][0] = pack_f16x2(bf16_lo(lo), bf16_hi(lo));
      qf[kk][1] = pack_f16x2(bf16_lo(hi), bf16_hi(hi));
      const float2 a = unpack_f16x2(qf[kk][0]), bb = unpack_f16x2(qf[kk][1]);
      part[kk / KK_PER_G] += (a.x + a.y) + (bb.x + bb.y);
    }
#pragma unroll
    for (int gr = 0; gr < NG; ++gr) {
      float v = part[gr];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);  // head g8's group sum, on its 4 lanes
      qsum[gr][0] = __shfl_sync(0xffffffffu, v, (2 * c4) * 4);
      qsum[gr][1] = __shfl_sync(0xffffffffu, v, (2 * c4 + 1) * 4);
    }
  }

  const int nj = n_here > warp ? (n_here - warp + NW - 1) / NW : 0;
  uint8_t* stage = smem + warp * NSTAGE * S::BLOCK;
  uint64_t* bar = bars + warp * NSTAGE;
  const int32_t* bt_row = block_table + (size_t)b * max_pages;
  auto issue = [&](int j) {
    int page = bt_row[p_begin + warp + j * NW];
    if (page < 0 || page >= num_pages) {
      flag_device(status, DEV_BAD_INDEX);
      page = 0;  // keep the copy in bounds; the status word reports the fault
    }
    const uint8_t* src = pool + ((size_t)page * Hkv + kvh) * S::BLOCK;
    const int s = j % NSTAGE;
    mbar_arrive_expect_tx(&bar[s], S::BLOCK);
    bulk_g2s(stage + s * S::BLOCK, src, S::BLOCK, &bar[s]);
  };
  int issued = 0;
  if (lane == 0)
    for (; issued < NSTAGE && issued < nj; ++issued) issue(issued);
  issued = __shfl_sync(0xffffffffu, issued, 0);

  float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F;
  float l0 = 0.f, l1 = 0.f;
  float o[S::KSTEPS][4];
#pragma unroll
  for (int mt = 0; mt < S::KSTEPS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float corr[NG][2];  // sum_t p vb - 1024 fp16(p vs), heads 2c, 2c+1 (this lane's tokens)
#pragma unroll
  for (int gr = 0; gr < NG; ++gr) corr[gr][0] = corr[gr][1] = 0.f;
  const int rot = 4 * g8;  // row rotation of K rows g8 and g8 + 8 (in words)
  int consumed = 0;
  for (int j = 0; j < nj; ++j) {
    const int s = j % NSTAGE;
    if (!mbar_wait_bounded(&bar[s], (j / NSTAGE) & 1, status)) break;
    const uint32_t base = smem_addr(stage + s * S::BLOCK);
    const int page_tok = (p_begin + warp + j * NW) * kPage;
    const int tok0 = page_tok + g8;
    const bool lo_ok = tok0 < L, hi_ok = tok0 + 8 < L;

    float acc[NG][4];
#pragma unroll
    for (int gr = 0; gr < NG; ++gr) acc[gr][0] = acc[gr][1] = acc[gr][2] = acc[gr][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < S::KSTEPS; ++kk) {
      const int pw = (4 * kk + c4 + rot) & (S::WORDS - 1);
      const uint32_t w0 = lds32(base + g8 * D + pw * 4);
      const uint32_t w1 = lds32(base + (g8 + 8) * D + pw * 4);
      mma_f16_16816(acc[kk / KK_PER_G], codes_lo(w0), codes_lo(w1), codes_hi(w0), codes_hi(w1),
                    qf[kk][0], qf[kk][1]);
    }
    float ks0[NG], ks1[NG], kb0[NG], kb1[NG];
    lds_bf16<NG>(base + S::OFF_KS + g8 * NG * 2, ks0);
    lds_bf16<NG>(base + S::OFF_KS + (g8 + 8) * NG * 2, ks1);
    lds_bf16<NG>(base + S::OFF_KB + g8 * NG * 2, kb0);
    lds_bf16<NG>(base + S::OFF_KB + (g8 + 8) * NG * 2, kb1);
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int gr = 0; gr < NG; ++gr) {
      const float b0 = kb0[gr] - 1024.f * ks0[gr], b1 = kb1[gr] - 1024.f * ks1[gr];
      sc[0] = fmaf(ks0[gr], acc[gr][0], fmaf(b0, qsum[gr][0], sc[0]));
      sc[1] = fmaf(ks0[gr], acc[gr][1], fmaf(b0, qsum[gr][1], sc[1]));
      sc[2] = fmaf(ks1[gr], acc[gr][2], fmaf(b1, qsum[gr][0], sc[2]));
      sc[3] = fmaf(ks1[gr], acc[gr][3], fmaf(b1, qsum[gr][1], sc[3]));
    }
    // Rows past the context: masked (their scale/bias bits may be anything).
    const float x0 = lo_ok ? sc[0] * scale_log2 : -CUDART_INF_F;
    const float x1 = lo_ok ? sc[1] * scale_log2 : -CUDART_INF_F;
    const float x2 = hi_ok ? sc[2] * scale_log2 : -CUDART_INF_F;
    const float x3 = hi_ok ? sc[3] * scale_log2 : -CUDART_INF_F;
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

    // Value side: probabilities scaled per group (rows past the context use 0
    // for scale and bias, so garbage bits there never reach the sums).
    float vs0[NG], vs1[NG], vb0[NG], vb1[NG];
    lds_bf16<NG>(base + S::OFF_VS + g8 * NG * 2, vs0);
    lds_bf16<NG>(base + S::OFF_VS + (g8 + 8) * NG * 2, vs1);
    lds_bf16<NG>(base + S::OFF_VB + g8 * NG * 2, vb0);
    lds_bf16<NG>(base + S::OFF_VB + (g8 + 8) * NG * 2, vb1);
    uint32_t pb[NG][2];
#pragma unroll
    for (int gr = 0; gr < NG; ++gr) {
      const float s0 = lo_ok ? vs0[gr] : 0.f, s1 = hi_ok ? vs1[gr] : 0.f;
      const float bb0 = lo_ok ? vb0[gr] : 0.f, bb1 = hi_ok ? vb1[gr] : 0.f;
      const uint32_t h01 = pack_f16x2(p0 * s0, p1 * s0);
      const uint32_t h23 = pack_f16x2(p2 * s1, p3 * s1);
      const float2 f01 = unpack_f16x2(h01), f23 = unpack_f16x2(h23);
      corr[gr][0] =
          fmaf(corr[gr][0], c0, fmaf(p0, bb0, fmaf(p2, bb1, -1024.f * (f01.x + f23.x))));
      corr[gr][1] =
          fmaf(corr[gr][1], c1, fmaf(p1, bb0, fmaf(p3, bb1, -1024.f * (f01.y + f23.y))));
      pb[gr][0] = movmatrix_t(h01);
      pb[gr][1] = movmatrix_t(h23);
    }
#pragma unroll
    for (int mt = 0; mt < S::KSTEPS; ++mt) {
      o[mt][0] *= c0;
      o[mt][1] *= c1;
      o[mt][2] *= c0;
      o[mt][3] *= c1;
      const uint32_t w0 = lds32(base + S::OFF_V + (16 * mt + g8) * 16 + c4 * 4);
      const uint32_t w1 = lds32(base + S::OFF_V + (16 * mt + g8 + 8) * 16 + c4 * 4);
      const int gr = mt / KK_PER_G;
      mma_f16_16816(o[mt], codes_lo(w0), codes_lo(w1), codes_hi(w0), codes_hi(w1), pb[gr][0],
                    pb[gr][1]);
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
    // A wait gave up (already flagged): drain this warp's copies in flight.
    for (int j = consumed; j < issued; ++j)
      if (!mbar_wait_bounded(&bar[j % NSTAGE], (j / NSTAGE) & 1, status)) break;
  }

  // The per-group value corrections: sum over the lanes of each head pair.
#pragma unroll
  for (int gr = 0; gr < NG; ++gr) {
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      corr[gr][0] += __shfl_xor_sync(0xffffffffu, corr[gr][0], off);
      corr[gr][1] += __shfl_xor_sync(0xffffffffu, corr[gr][1], off);
    }
  }
#pragma unroll
  for (int mt = 0; mt < S::KSTEPS; ++mt) {
    const int gr = mt / KK_PER_G;
    o[mt][0] += corr[gr][0];
    o[mt][1] += corr[gr][1];
    o[mt][2] += corr[gr][0];
    o[mt][3] += corr[gr][1];
  }
#pragma unroll
  for (int off = 4; off <= 16; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  __syncthreads();  // every stage is drained; reuse the stage memory

  float* red_o = reinterpret_cast<float*>(smem);  // [NW][8][D]
  float* red_m = red_o + NW * kHeadsPerTile * D;  // [NW][8]
  float* red_l = red_m + NW * kHeadsPerTile;      // [NW][8]
  {
    const int h0 = 2 * c4;
    float* w0 = red_o + (warp * kHeadsPerTile + h0) * D;
    float* w1 = w0 + D;
#pragma unroll
    for (int mt = 0; mt < S::KSTEPS; ++mt) {
      w0[16 * mt + g8] = o[mt][0];
      w1[16 * mt + g8] = o[mt][1];
      w0[16 * mt + g8 + 8] = o[mt][2];
      w1[16 * mt + g8 + 8] = o[mt][3];
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
    float lsum = 0.f, accv = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float mw = red_m[w * kHeadsPerTile + n];
      const float f = mw == -CUDART_INF_F ? 0.f : exp2f(mw - M);
      lsum = fmaf(red_l[w * kHeadsPerTile + n], f, lsum);
      accv = fmaf(red_o[(w * kHeadsPerTile + n) * D + d], f, accv);
    }
    const float val = accv / lsum;
    const float lse = (M + log2f(lsum)) * kLn2;
    const size_t row = (size_t)b * Hq + head0 + n;
    if (num_splits == 1) {
      out[row * D + d] = f_to_bf16(val);
      if (d == 0 && lse_out != nullptr) lse_out[row] = lse;
    } else {
      part_out[(row * num_splits + split) * D + d] = val;
      if (d == 0) part_lse[row * num_splits + split] = lse;
    }
  }
}

// Launch shape: warps per CTA and shared-memory stages (one page block each) per warp.
#ifndef SC_Q8_WARPS
#define SC_Q8_WARPS 4
#endif
#ifndef SC_Q8_STAGES
#define SC_Q8_STAGES 2  // 70 KiB CTAs, three per SM: 90% of measured HBM on config 3
#endif
constexpr int kQ8Warps = SC_Q8_WARPS, kQ8Stages = SC_Q8_STAGES;

template <int D>
int launch_q8(const uint16_t* q, const uint8_t* pool, const int32_t* block_table,
              const int32_t* ctx_len, const int32_t* seq_order, int B, int Hq, int Hkv, int max_pages, int pages_per_split,
              int num_splits, float scale, float* part_out, float* part_lse, uint16_t* out,
              float* lse_out, long long num_pages, cudaStream_t s) {
  using S = Q8<D>;
  constexpr int NW = kQ8Warps, NST = kQ8Stages;
  const size_t smem_stages = (size_t)NW * NST * S::BLOCK + NW * NST * sizeof(uint64_t);
  const size_t smem_merge = (size_t)NW * kHeadsPerTile * (D + 2) * sizeof(float);
  const size_t smem = smem_stages > smem_merge ? smem_stages : smem_merge;
  auto kernel = paged_decode_q8_kernel<D, NW, NST>;
  static int configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t err =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess)
      return set_error(SC_ERR_CUDA, "sc_paged_decode_attention_q8: smem attribute: %s",
                       cudaGetErrorString(err));
    configured[dev] = 1;
  }
  const int G = Hq / Hkv;
  const int HG = (G + kHeadsPerTile - 1) / kHeadsPerTile;
  dim3 grid(num_splits, Hkv * HG, B);
  kernel<<<grid, NW * 32, smem, s>>>(q, pool, block_table, ctx_len, seq_order, Hq, Hkv, G, HG,
                                     max_pages,
                                     pages_per_split, num_splits, scale * 1.4426950408889634f,
                                     part_out, part_lse, out, lse_out, num_pages,
                                     device_status_word());
  if (int rc = check_launch("sc_paged_decode_attention_q8")) return rc;
  if (num_splits > 1) {
    launch_combine(part_out, part_lse, (size_t)num_splits * D, D, num_splits, 1, ctx_len, Hq,
                   num_splits, pages_per_split, D, B * Hq, out, lse_out, nullptr, s);
    return check_launch("sc_paged_decode_attention_q8(combine)");
  }
  return SC_OK;
}

// Page copies (copy-on-write of a shared prefix page) for 8-bit pools.
__global__ void q8_copy_pages_kernel(uint4* __restrict__ pool, const int32_t* __restrict__ src,
                                     const int32_t* __restrict__ dst, long long total,
                                     int page_chunks, long long num_pages, unsigned int* status) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const long long i = idx / page_chunks;
  const int c = (int)(idx - i * page_chunks);
  const int32_t a = src[i], b = dst[i];
  if (a < 0 || b < 0 || a >= num_pages || b >= num_pages) {
    flag_device(status, DEV_BAD_INDEX);
    return;
  }
  pool[(size_t)b * page_chunks + c] = pool[(size_t)a * page_chunks + c];
}

int check_q8_pool(const char* name, int Hkv, int D, int P, long long num_pages) {
  SC_REQUIRE(Hkv > 0 && num_pages > 0, SC_ERR_INVALID, "%s: Hkv=%d num_pages=%lld", name, Hkv,
             num_pages);
  SC_REQUIRE(D == 128 || D == 256, SC_ERR_UNSUPPORTED, "%s: D=%d not in {128, 256}", name, D);
  SC_REQUIRE(P == kPage, SC_ERR_UNSUPPORTED, "%s: page size %d != 16", name, P);
  return SC_OK;
}

}  // namespace
}  // namespace sc

extern "C" int sc_kv_q8_block_bytes(int D) {
  return (D == 128 || D == 256) ? sc::q8_block_bytes(D) : 0;
}

extern "C" int sc_kv_append_q8(const sc_bf16* k, const sc_bf16* v, uint8_t* kv_pool,
                               const int64_t* slot_mapping, int ntok, int Hkv, int D, int P,
                               int64_t num_pages, void* stream) {
  using namespace sc;
  const char* name = "sc_kv_append_q8";
  if (int rc = check_q8_pool(name, Hkv, D, P, num_pages)) return rc;
  SC_REQUIRE(k && v && kv_pool && slot_mapping, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(ntok >= 0, SC_ERR_INVALID, "%s: ntok=%d", name, ntok);
  if (ntok == 0) return SC_OK;
  const long long threads = (long long)ntok * Hkv * 2 * 32;
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 128)
    kv_append_q8_kernel<128><<<blocks, 256, 0, s>>>(k, v, kv_pool, slot_mapping, ntok, Hkv,
                                                    num_pages, device_status_word());
  else
    kv_append_q8_kernel<256><<<blocks, 256, 0, s>>>(k, v, kv_pool, slot_mapping, ntok, Hkv,
                                                    num_pages, device_status_word());
  return check_launch(name);
}

extern "C" int sc_kv_gather_q8(const uint8_t* kv_pool, const int64_t* slot_mapping, int ntok,
                               int Hkv, int D, int P, int64_t num_pages, uint8_t* codes,
                               sc_bf16* scale_bias, void* stream) {
  using namespace sc;
  const char* name = "sc_kv_gather_q8";
  if (int rc = check_q8_pool(name, Hkv, D, P, num_pages)) return rc;
  SC_REQUIRE(kv_pool && slot_mapping && codes && scale_bias, SC_ERR_INVALID, "%s: null pointer",
             name);
  SC_REQUIRE(ntok >= 0, SC_ERR_INVALID, "%s: ntok=%d", name, ntok);
  if (ntok == 0) return SC_OK;
  const long long total = (long long)ntok * Hkv * 2 * D;
  const unsigned blocks = (unsigned)((total + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 128)
    kv_gather_q8_kernel<128><<<blocks, 256, 0, s>>>(kv_pool, slot_mapping, ntok, Hkv, num_pages,
                                                    codes, scale_bias, device_status_word());
  else
    kv_gather_q8_kernel<256><<<blocks, 256, 0, s>>>(kv_pool, slot_mapping, ntok, Hkv, num_pages,
                                                    codes, scale_bias, device_status_word());
  return check_launch(name);
}

extern "C" int sc_kv_copy_pages_q8(uint8_t* kv_pool, const int32_t* src, const int32_t* dst,
                                   int npages, int Hkv, int D, int P, int64_t num_pages,
                                   void* stream) {
  using namespace sc;
  const char* name = "sc_kv_copy_pages_q8";
  if (int rc = check_q8_pool(name, Hkv, D, P, num_pages)) return rc;
  SC_REQUIRE(kv_pool && src && dst, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(npages >= 0, SC_ERR_INVALID, "%s: npages=%d", name, npages);
  SC_REQUIRE((reinterpret_cast<uintptr_t>(kv_pool) & 15) == 0, SC_ERR_INVALID,
             "%s: kv_pool must be 16-byte aligned", name);
  if (npages == 0) return SC_OK;
  const int page_chunks = Hkv * q8_block_bytes(D) / 16;
  const long long total = (long long)npages * page_chunks;
  q8_copy_pages_kernel<<<(unsigned)((total + 255) / 256), 256, 0,
                         static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<uint4*>(kv_pool), src, dst, total, page_chunks, num_pages,
      device_status_word());
  return check_launch(name);
}

extern "C" int sc_paged_decode_attention_q8(const sc_bf16* q, const uint8_t* kv_pool,
                                            int64_t num_pages, const int32_t* block_table,
                                            const int32_t* ctx_len, const int32_t* seq_order,
                                            int B, int Hq, int Hkv, int D, int P, int max_pages,
                                            int pages_per_split,
                                            int num_splits, float scale, float* part_out,
                                            float* part_lse, sc_bf16* out, float* lse_out,
                                            void* stream) {
  using namespace sc;
  const char* name = "sc_paged_decode_attention_q8";
  if (int rc = check_q8_pool(name, Hkv, D, P, num_pages)) return rc;
  SC_REQUIRE(q && kv_pool && block_table && ctx_len && out, SC_ERR_INVALID, "%s: null pointer",
             name);
  SC_REQUIRE(B >= 0 && Hq > 0 && Hq % Hkv == 0, SC_ERR_INVALID, "%s: bad heads Hq=%d Hkv=%d",
             name, Hq, Hkv);
  SC_REQUIRE(max_pages > 0 && pages_per_split > 0 && num_splits > 0, SC_ERR_INVALID,
             "%s: bad split plan max_pages=%d pages_per_split=%d num_splits=%d", name, max_pages,
             pages_per_split, num_splits);
  SC_REQUIRE(num_splits == 1 || (part_out && part_lse), SC_ERR_INVALID,
             "%s: num_splits > 1 needs part_out and part_lse", name);
  SC_REQUIRE(num_splits <= 65535 && B <= 65535 && Hkv * ((Hq / Hkv + 7) / 8) <= 65535,
             SC_ERR_INVALID, "%s: grid too large", name);
  SC_REQUIRE((reinterpret_cast<uintptr_t>(kv_pool) & 15) == 0, SC_ERR_INVALID,
             "%s: kv_pool must be 16-byte aligned", name);
  if (B == 0) return SC_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 128)
    return launch_q8<128>(q, kv_pool, block_table, ctx_len, seq_order, B, Hq, Hkv, max_pages,
                          pages_per_split, num_splits, scale, part_out, part_lse, out, lse_out,
                          num_pages, s);
  return launch_q8<256>(q, kv_pool, block_table, ctx_len, seq_order, B, Hq, Hkv, max_pages,
                        pages_per_split, num_splits, scale, part_out, part_lse, out, lse_out,
                        num_pages, s);
}
