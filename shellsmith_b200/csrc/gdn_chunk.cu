// K2+K3 gdn_chunk_prefill: chunk-64 gated-delta prefill on tcgen05 tensor cores.
//
// Reference: studio_compute/numerics/ops.py:151-215 `gated_delta_chunked`
// (WY/UT chunk form, _invert_unit_lower :54-85, _scan_forward :88-104) and the
// fused Metal path numerics/gdn_fused.py:86-171. Per chunk of C = 64 tokens,
// with lg = cumsum(log clamp(g, 1e-6, 1)), decay = e^lg, R_tj = e^(lg_t - lg_j),
// r_t = e^(lg_63 - lg_t), A_tj = beta_t R_tj (k_t . k_j) (j < t), X = (I + A)^-1,
// m_tj = R_tj (q_t . k_j) (j <= t), the reference computes u0 = X(beta v),
// kt = X(beta decay k), q_eff = decay q - m kt, mu0 = m u0 and scans
//   O = mu0 + q_eff S^T,  U = u0 - kt S^T,  S <- decay_63 S + (r U)^T K.
// Substituting gives the same numbers with two fewer products:
//   W = beta (V - decay (K S^T)),  U = X W,  O = decay (Q S^T) + (m X) W,
//   S <- decay_63 S + (r U)^T K.
//
// B200 mapping. One CTA (4 warps) owns one (sequence, value head) and walks its
// chunks in order; the 128 x 128 fp32 state lives in tensor memory the whole
// time. Everything is computed transposed, so TMEM lane = value row i = thread:
//   G0  [K;Q] K^T            -> A (fp32 smem), m        M128 N64  K128
//   Y   m X                  -> rows 64.. of [X;Y]      M128 N64  K64
//   G12 S [K;Q]^T            -> P1^T | P2^T             M128 N128 K128
//   G34 W^T [X;Y]^T (+= 0 | decay P2^T) -> U^T | O^T    M128 N128 K64
//   GS  (U^T r) K  (+= decay_63 S)                      M128 N128 K64
// Q/K/V chunk tiles arrive by TMA (128-byte swizzle, no multicast); the
// unit-lower inverse runs column-per-thread in fp32. Operands that feed the
// fp32 state (S, W, X, Y, U) are split into bf16 hi + lo and multiplied as
// hi*hi + hi*lo + lo*hi, which keeps the state within ~1e-5 of fp32 math.
#include <cudaTypedefs.h>
#include <math_constants.h>

#include <mutex>

#include "tc.cuh"

namespace sc {
namespace {

constexpr int kC = 64;    // chunk length
constexpr int kD = 128;   // key and value width
constexpr int kThreads = 128;

// Shared memory plan (byte offsets from a 1024-aligned base).
constexpr uint32_t OFF_KQ = 0;          // [2 dk halves][K rows 0-63 | Q rows 64-127][128 B]
constexpr uint32_t OFF_V = 32768;       // [2 dv halves][64 rows][128 B]
constexpr uint32_t OFF_SH = 49152;      // S hi  [2 dk blocks][128 rows][128 B]
constexpr uint32_t OFF_SL = 81920;      // S lo
constexpr uint32_t OFF_XYH = 114688;    // [X rows 0-63 | Y rows 64-127][128 B] hi
constexpr uint32_t OFF_XYL = 131072;    // lo
constexpr uint32_t OFF_WH = 147456;     // W^T hi, later (U^T r) hi [128 rows][128 B]
constexpr uint32_t OFF_WL = 163840;     // lo
constexpr uint32_t OFF_SMALL = 180224;  // lg, beta, decay, r [64] floats; barriers; TMEM base
// Aliases used while a chunk is prepared (regions free at that time):
constexpr uint32_t OFF_MH = OFF_SH;            // m hi [128 rows (0-63 used)][128 B]
constexpr uint32_t OFF_ML = OFF_SH + 16384;    // m lo
constexpr uint32_t OFF_AMAT = OFF_SH + 32768;  // A (strict lower) fp32 [64][68]
constexpr uint32_t OFF_XTH = OFF_WH;           // X^T rows hi [64 rows][128 B]
constexpr uint32_t OFF_XTL = OFF_WL;           // lo
constexpr int kAStride = 68;                   // fp32 row stride of A (conflict-free float4 rows)
constexpr uint32_t SMEM_BYTES = OFF_SMALL + 4 * 64 * 4 + 32 + 1024;  // + 1024 alignment slack

// TMEM columns (512 allocated).
constexpr uint32_t T_S = 0, T_P = 128, T_KK = 256, T_Y = 320;

__device__ __forceinline__ void store_chunks_hilo(uint8_t* hi, uint8_t* lo, int row, int c0,
                                                  const float* x) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = x[8 * c + 2 * e], b = x[8 * c + 2 * e + 1];
      h[e] = pack_bf16x2(a, b);
      l[e] = pack_bf16x2(a - bf16_lo(h[e]), b - bf16_hi(h[e]));
    }
    const uint32_t off = (uint32_t)row * 128u + (uint32_t)((((c0 + c) ^ (row & 7)) << 4));
    *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    gdn_chunk_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const float* __restrict__ g,
                     const float* __restrict__ beta, float* __restrict__ state,
                     const int32_t* __restrict__ state_slot,
                     const int32_t* __restrict__ cu_seqlens, uint16_t* __restrict__ out, int Hk,
                     int Hv, int T_fixed, int num_slots, unsigned int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~uintptr_t(1023));
  float* s_lg = reinterpret_cast<float*>(sm + OFF_SMALL);
  float* s_beta = s_lg + 64;
  float* s_decay = s_beta + 64;
  float* s_r = s_decay + 64;
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(s_r + 64);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bar_mma + 1);

  const int bh = blockIdx.x;
  const int b = bh / Hv;
  const int h = bh - b * Hv;
  const int kh = h / (Hv / Hk);
  const int start = cu_seqlens != nullptr ? cu_seqlens[b] : b * T_fixed;
  const int len = cu_seqlens != nullptr ? cu_seqlens[b + 1] - start : T_fixed;
  const int slot = state_slot != nullptr ? state_slot[b] : b;
  if (slot < 0 || len <= 0) return;  // uniform over the CTA
  if (slot >= num_slots) {
    if (threadIdx.x == 0) flag_device(status, DEV_BAD_INDEX);
    return;
  }
  // After any bounded wait has given up on this device, later CTAs stop at once.
  if (status != nullptr && (*reinterpret_cast<volatile unsigned int*>(status) & DEV_WAIT_TIMEOUT))
    return;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int i = tid;  // value row = TMEM lane

  if (tid == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(s_tmem, 512);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *s_tmem;
  const uint32_t lane = (uint32_t)(warp * 32) << 16;

  // Initial state row i -> TMEM.
  float* srow = state + ((size_t)slot * Hv + h) * kD * kD + (size_t)i * kD;
#pragma unroll 1
  for (int q = 0; q < 4; ++q) {
    float v[32];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float4 x = reinterpret_cast<const float4*>(srow + 32 * q)[e];
      v[4 * e] = x.x;
      v[4 * e + 1] = x.y;
      v[4 * e + 2] = x.z;
      v[4 * e + 3] = x.w;
    }
    tc::tmem_st32(tmem + lane + T_S + 32 * q, v);
  }
  tc::tmem_wait_st();

  uint32_t tma_phase = 0, mma_phase = 0;
  int ok = 1;
  int pending_tma = 0, pending_mma = 0;
  const int nchunks = (len + kC - 1) / kC;
  auto wait_mma = [&]() {
    int done = mbar_wait_bounded(bar_mma, mma_phase, status) ? 1 : 0;
    if (done) {
      mma_phase ^= 1;
    }
    ok = __syncthreads_and(done && ok);
    if (ok) pending_mma = 0;
    tc::fence_after();
    return ok;
  };

#pragma unroll 1
  for (int c = 0; c < nchunks; ++c) {
    const int tok0 = start + c * kC;
    const int valid = min(kC, len - c * kC);

    // ---- (1) chunk tiles by TMA; gates on the CUDA cores meanwhile.
    if (tid == 0) {
      mbar_arrive_expect_tx(bar_tma, 6 * 8192);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tc::tma_load_3d(sm + OFF_KQ + half * 16384, &tm_k, half * 64, kh, tok0, bar_tma);
        tc::tma_load_3d(sm + OFF_KQ + half * 16384 + 8192, &tm_q, half * 64, kh, tok0, bar_tma);
        tc::tma_load_3d(sm + OFF_V + half * 8192, &tm_v, half * 64, h, tok0, bar_tma);
      }
    }
    pending_tma = 1;
    if (tid < 64) {
      const bool on = tid < valid;
      const float gv = on ? g[(size_t)(tok0 + tid) * Hv + h] : 1.f;
      s_beta[tid] = on ? beta[(size_t)(tok0 + tid) * Hv + h] : 0.f;
      float lg = logf(fminf(fmaxf(gv, 1e-6f), 1.f));
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, lg, off);
        if ((tid & 31) >= off) lg += y;
      }
      s_lg[tid] = lg;
    }
    __syncthreads();
    if (tid >= 32 && tid < 64) s_lg[tid] += s_lg[31];
    __syncthreads();
    if (tid < 64) {
      s_decay[tid] = expf(s_lg[tid]);
      s_r[tid] = expf(s_lg[63] - s_lg[tid]);
    }
    {
      const int done = mbar_wait_bounded(bar_tma, tma_phase, status) ? 1 : 0;
      if (done) tma_phase ^= 1;
      ok = __syncthreads_and(done && ok);
      if (!ok) break;
      pending_tma = 0;
    }

    // ---- (2) G0: [K;Q] K^T -> TMEM cols T_KK (lanes 0-63 KK^T, 64-127 QK^T).
    if (tid == 0) {
      tc::fence_after();
      constexpr uint32_t id = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
      for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t a = smem_addr(sm + OFF_KQ + kb * 16384) + ks * 32;
          tc::mma_bf16(tmem + T_KK, tc::desc_kmajor(a), tc::desc_kmajor(a), id, (kb | ks) != 0);
        }
      tc::commit(bar_mma);
    }
    pending_mma = 1;
    if (!wait_mma()) break;

    // ---- (3) rows t of A (warps 0-1) and of m (warps 2-3).
    {
      float row[64];
      tc::tmem_ld32(tmem + lane + T_KK, row);
      tc::tmem_ld32(tmem + lane + T_KK + 32, row + 32);
      const int t = tid & 63;
      const float lgt = s_lg[t];
      if (warp < 2) {
        const float bt = s_beta[t];
        float4* arow = reinterpret_cast<float4*>(sm + OFF_AMAT) + t * (kAStride / 4);
#pragma unroll
        for (int j4 = 0; j4 < 16; ++j4) {
          float4 a;
          const int j = 4 * j4;
          a.x = j + 0 < t ? bt * expf(lgt - s_lg[j + 0]) * row[j + 0] : 0.f;
          a.y = j + 1 < t ? bt * expf(lgt - s_lg[j + 1]) * row[j + 1] : 0.f;
          a.z = j + 2 < t ? bt * expf(lgt - s_lg[j + 2]) * row[j + 2] : 0.f;
          a.w = j + 3 < t ? bt * expf(lgt - s_lg[j + 3]) * row[j + 3] : 0.f;
          arow[j4] = a;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) row[j] = j <= t ? expf(lgt - s_lg[j]) * row[j] : 0.f;
        tc::store_row_hilo(sm + OFF_MH, sm + OFF_ML, t, row);
      }
    }
    __syncthreads();

    // ---- (4) X = (I + A)^-1, column j per thread (warps 0-1).
    if (warp < 2) {
      const int j = tid;
      const float* A = reinterpret_cast<const float*>(sm + OFF_AMAT);
      float x[64];
#pragma unroll
      for (int t = 0; t < 64; ++t) {
        float acc = (t == j) ? 1.f : 0.f;
#pragma unroll
        for (int k = 0; k < t; ++k) acc = fmaf(-A[t * kAStride + k], x[k], acc);
        x[t] = acc;
      }
      tc::store_row_hilo(sm + OFF_XTH, sm + OFF_XTL, j, x);  // X^T row j
#pragma unroll
      for (int t = 0; t < 64; ++t) {                           // X rows, column j
        const uint16_t hi = f_to_bf16(x[t]);
        const uint16_t lo = f_to_bf16(x[t] - bf16_to_f(hi));
        *reinterpret_cast<uint16_t*>(sm + OFF_XYH + tc::swz(t, j)) = hi;
        *reinterpret_cast<uint16_t*>(sm + OFF_XYL + tc::swz(t, j)) = lo;
      }
    }
    fence_proxy_async_smem();
    __syncthreads();

    // ---- (5) Y = m X -> TMEM cols T_Y (lanes 0-63).
    if (tid == 0) {
      tc::fence_after();
      constexpr uint32_t id = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint64_t mh = tc::desc_kmajor(smem_addr(sm + OFF_MH) + ks * 32);
        const uint64_t ml = tc::desc_kmajor(smem_addr(sm + OFF_ML) + ks * 32);
        const uint64_t xh = tc::desc_kmajor(smem_addr(sm + OFF_XTH) + ks * 32);
        const uint64_t xl = tc::desc_kmajor(smem_addr(sm + OFF_XTL) + ks * 32);
        tc::mma_bf16(tmem + T_Y, mh, xh, id, ks != 0);
        tc::mma_bf16(tmem + T_Y, mh, xl, id, true);
        tc::mma_bf16(tmem + T_Y, ml, xh, id, true);
      }
      tc::commit(bar_mma);
    }
    pending_mma = 1;
    if (!wait_mma()) break;
    if (warp < 2) {
      float y[64];
      tc::tmem_ld32(tmem + lane + T_Y, y);
      tc::tmem_ld32(tmem + lane + T_Y + 32, y + 32);
      tc::store_row_hilo(sm + OFF_XYH, sm + OFF_XYL, 64 + tid, y);
    }

    // ---- (6) S hi/lo -> smem (A of G12); decay_63 * S -> TMEM.
    {
      const float dl = s_decay[63];
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
        float v[32];
        tc::tmem_ld32(tmem + lane + T_S + 32 * q, v);
        const uint32_t kb = (uint32_t)(q >> 1) * 16384u;
        store_chunks_hilo(sm + OFF_SH + kb, sm + OFF_SL + kb, i, 4 * (q & 1), v);
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] *= dl;
        tc::tmem_st32(tmem + lane + T_S + 32 * q, v);
      }
      tc::tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc::fence_before();
    __syncthreads();

    // ---- (7) G12: S [K;Q]^T -> TMEM cols T_P.
    if (tid == 0) {
      tc::fence_after();
      constexpr uint32_t id = tc::idesc_bf16(128, 128, false, false);
#pragma unroll
      for (int part = 0; part < 2; ++part)
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint32_t a = smem_addr(sm + (part ? OFF_SL : OFF_SH) + kb * 16384) + ks * 32;
            const uint32_t bb = smem_addr(sm + OFF_KQ + kb * 16384) + ks * 32;
            tc::mma_bf16(tmem + T_P, tc::desc_kmajor(a), tc::desc_kmajor(bb), id,
                         (part | kb | ks) != 0);
          }
      tc::commit(bar_mma);
    }
    pending_mma = 1;
    if (!wait_mma()) break;

    // ---- (8) W^T row i; zero U^T columns; decay * P2^T in the O^T columns.
    {
      float p[64];
      tc::tmem_ld32(tmem + lane + T_P, p);
      tc::tmem_ld32(tmem + lane + T_P + 32, p + 32);
      const uint8_t* vt = sm + OFF_V + (i >> 6) * 8192;
      const int iv = i & 63;
#pragma unroll
      for (int t = 0; t < 64; ++t) {
        const float vti = bf16_to_f(*reinterpret_cast<const uint16_t*>(vt + tc::swz(t, iv)));
        p[t] = s_beta[t] * (vti - s_decay[t] * p[t]);
      }
      tc::store_row_hilo(sm + OFF_WH, sm + OFF_WL, i, p);
      float z[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) z[e] = 0.f;
      tc::tmem_st32(tmem + lane + T_P, z);
      tc::tmem_st32(tmem + lane + T_P + 32, z);
      tc::tmem_ld32(tmem + lane + T_P + 64, p);
      tc::tmem_ld32(tmem + lane + T_P + 96, p + 32);
#pragma unroll
      for (int t = 0; t < 64; ++t) p[t] *= s_decay[t];
      tc::tmem_st32(tmem + lane + T_P + 64, p);
      tc::tmem_st32(tmem + lane + T_P + 96, p + 32);
      tc::tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc::fence_before();
    __syncthreads();

    // ---- (9) G34: W^T [X;Y]^T accumulated -> U^T | O^T.
    if (tid == 0) {
      tc::fence_after();
      constexpr uint32_t id = tc::idesc_bf16(128, 128, false, false);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint64_t wh = tc::desc_kmajor(smem_addr(sm + OFF_WH) + ks * 32);
        const uint64_t wl = tc::desc_kmajor(smem_addr(sm + OFF_WL) + ks * 32);
        const uint64_t xh = tc::desc_kmajor(smem_addr(sm + OFF_XYH) + ks * 32);
        const uint64_t xl = tc::desc_kmajor(smem_addr(sm + OFF_XYL) + ks * 32);
        tc::mma_bf16(tmem + T_P, wh, xh, id, true);
        tc::mma_bf16(tmem + T_P, wh, xl, id, true);
        tc::mma_bf16(tmem + T_P, wl, xh, id, true);
      }
      tc::commit(bar_mma);
    }
    pending_mma = 1;
    if (!wait_mma()) break;

    // ---- (10) O^T -> out (bf16); (U^T r) hi/lo -> smem (A of GS).
    {
      float u[64];
      tc::tmem_ld32(tmem + lane + T_P + 64, u);
      tc::tmem_ld32(tmem + lane + T_P + 96, u + 32);
      uint16_t* orow = out + ((size_t)tok0 * Hv + h) * kD + i;
#pragma unroll
      for (int t = 0; t < 64; ++t)
        if (t < valid) orow[(size_t)t * Hv * kD] = f_to_bf16(u[t]);
      tc::tmem_ld32(tmem + lane + T_P, u);
      tc::tmem_ld32(tmem + lane + T_P + 32, u + 32);
#pragma unroll
      for (int t = 0; t < 64; ++t) u[t] *= s_r[t];
      tc::store_row_hilo(sm + OFF_WH, sm + OFF_WL, i, u);
    }
    fence_proxy_async_smem();
    tc::fence_before();
    __syncthreads();

    // ---- (11) GS: S += (U^T r) K, K as an MN-major operand (dk halves 16 KiB apart).
    if (tid == 0) {
      tc::fence_after();
      constexpr uint32_t id = tc::idesc_bf16(128, 128, false, true);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint64_t kd = tc::desc_mnmajor(smem_addr(sm + OFF_KQ) + ks * 2048, 16384);
        tc::mma_bf16(tmem + T_S, tc::desc_kmajor(smem_addr(sm + OFF_WH) + ks * 32), kd, id, true);
        tc::mma_bf16(tmem + T_S, tc::desc_kmajor(smem_addr(sm + OFF_WL) + ks * 32), kd, id, true);
      }
      tc::commit(bar_mma);
    }
    pending_mma = 1;
    if (!wait_mma()) break;
  }

  if (!ok) {
    // A bounded wait gave up (already flagged): let this CTA's own copies and
    // MMAs in flight finish, within limits, before the TMEM is released.
    if (pending_tma) mbar_wait_bounded(bar_tma, tma_phase, status);
    if (pending_mma) mbar_wait_bounded(bar_mma, mma_phase, status);
  } else {
#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
      float v[32];
      tc::tmem_ld32(tmem + lane + T_S + 32 * q, v);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        reinterpret_cast<float4*>(srow + 32 * q)[e] =
            make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// [tokens][heads][128] bf16 viewed as a 3-D tensor (d, head, token); box 64 x 1 x 64.
int encode_rows(CUtensorMap* map, const void* base, int heads, long long tokens,
                const char* what) {
  auto fn = encode_fn();
  if (fn == nullptr)
    return set_error(SC_ERR_CUDA, "sc_gdn_chunk_prefill: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)heads, (cuuint64_t)tokens};
  cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)heads * kD * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)kC};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                  strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(SC_ERR_INVALID, "sc_gdn_chunk_prefill: tensor map for %s rejected (%d)",
                     what, (int)r);
  return SC_OK;
}

}  // namespace
}  // namespace sc

extern "C" int sc_gdn_chunk_prefill(const sc_bf16* q, const sc_bf16* k, const sc_bf16* v,
                                    const float* g, const float* beta, float* state,
                                    const int32_t* state_slot, const int32_t* cu_seqlens,
                                    sc_bf16* out, int B, int T, int total_tokens, int Hk, int Hv,
                                    int dk, int dv, int num_slots, void* stream) {
  const char* name = "sc_gdn_chunk_prefill";
  SC_REQUIRE(q && k && v && g && beta && state && out, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(dk == sc::kD && dv == sc::kD, SC_ERR_UNSUPPORTED, "%s: dk=%d dv=%d (only 128x128)",
             name, dk, dv);
  SC_REQUIRE(B >= 0 && Hk > 0 && Hv > 0 && Hv % Hk == 0, SC_ERR_INVALID,
             "%s: bad heads B=%d Hk=%d Hv=%d", name, B, Hk, Hv);
  SC_REQUIRE((long long)B * Hv < (1LL << 31), SC_ERR_INVALID, "%s: B*Hv too large", name);
  SC_REQUIRE(num_slots > 0 && (state_slot != nullptr || num_slots >= B), SC_ERR_INVALID,
             "%s: num_slots=%d for B=%d", name, num_slots, B);
  long long tokens;
  if (cu_seqlens == nullptr) {
    SC_REQUIRE(T >= 0, SC_ERR_INVALID, "%s: T=%d", name, T);
    tokens = (long long)B * T;
  } else {
    SC_REQUIRE(total_tokens >= 0, SC_ERR_INVALID, "%s: total_tokens=%d", name, total_tokens);
    tokens = total_tokens;
  }
  if (B == 0 || tokens == 0) return SC_OK;
  SC_REQUIRE(tokens < (1LL << 31), SC_ERR_INVALID, "%s: too many tokens", name);
  SC_REQUIRE(((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16 == 0, SC_ERR_INVALID,
             "%s: q/k/v must be 16-byte aligned", name);
  CUtensorMap tq, tk, tv;
  if (int rc = sc::encode_rows(&tq, q, Hk, tokens, "q")) return rc;
  if (int rc = sc::encode_rows(&tk, k, Hk, tokens, "k")) return rc;
  if (int rc = sc::encode_rows(&tv, v, Hv, tokens, "v")) return rc;

  static int configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t err = cudaFuncSetAttribute(sc::gdn_chunk_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)sc::SMEM_BYTES);
    if (err != cudaSuccess)
      return sc::set_error(SC_ERR_CUDA, "%s: smem attribute: %s", name, cudaGetErrorString(err));
    configured[dev] = 1;
  }
  sc::gdn_chunk_kernel<<<B * Hv, sc::kThreads, sc::SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(
      tq, tk, tv, g, beta, state, state_slot, cu_seqlens, out, Hk, Hv, T, num_slots,
      sc::device_status_word());
  return sc::check_launch(name);
}
