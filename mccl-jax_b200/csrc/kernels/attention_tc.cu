// attention_tc.cu — fused softmax(scale * Q K^T [causal]) V on the B200 tensor cores, bf16 in/out,
// fp32 scores / softmax / accumulation.
//
// The reference runs attention as three MPSGraph ops with the full S x S score matrix in memory:
// DotGeneral (src/jam/ops/linalg.mm:98), the softmax pattern match (src/jam/ops/elementwise.mm:71-89)
// and a second DotGeneral.  Here the whole chain is one kernel and the scores never leave the SM.
//
// CTA = two 128-row query tiles of one (batch, head) = 256 queries; KV tiles of 128 keys.
//   warps 0-3   softmax warpgroup for query tile 0 (thread i owns query row i = TMEM lane i)
//   warps 4-7   softmax warpgroup for query tile 1
//   warp 8      TMA loads: Q0, Q1 once; K_j and V_j through two-stage rings
//   warp 9      allocates 512 TMEM columns; one thread issues every tcgen05.mma
// TMEM: S_t (128 x 128 f32) at column 128 t, O_t (128 x D f32) at column 256 + D t, and P_t
// (128 x 128 bf16, two per 32-bit column) at column 256 + 2 D + 64 t.
// Per KV tile j and query tile t:
//   S_t = Q_t K_j^T (tensor core)  ->  the softmax warps load their S row once, release S_t, take
//   the row max (four independent chains), write P_t = exp2(s - m) as bf16 into tensor memory
//   (tcgen05.st; the row sums in four independent packed accumulators)  ->  O_t += P_t V_j (tensor
//   core, A operand read from tensor memory, accumulating in TMEM).
// The running max used for P only moves when the true row max exceeds it by more than 2^8
// (lazy rescaling): then the warp rescales its O row in TMEM (ld / scale / st) before the next
// P V product; otherwise O is never touched by the CUDA cores until the final 1 / l.
// Per KV tile the MMA thread issues both tiles' S_t(j+1) as soon as their softmax has read S_t(j),
// then both P V(j) products: the tensor core computes the next scores while the softmax runs, and
// neither softmax group waits behind the other's P.
// V is read in place ([B*H, S, D], D contiguous) as the MN-major B operand of the P V product; the
// VT variant (V pre-transposed to [B*H, D, S], K-major) and P in shared memory (PT = false, two
// buffers per tile, 128-byte swizzled, read through a descriptor) are kept as cross-checks.
#include <cuda_bf16.h>
#include <cstdlib>
#include <mutex>

#include "kernels.h"
#include "tc_common.cuh"
#include "../../../include/b200_kernels.h"

namespace b200k {

static __device__ int g_tc_error_attn;

namespace {

constexpr int TQ = 128, TK = 128;
constexpr float kRescaleThreshold = 8.0f;   // log2 units: P entries stay <= 256

template <int D>
struct ACfg {
  static constexpr int kQBytes = TQ * D * 2;          // one query tile
  static constexpr int kKBytes = TK * D * 2;          // one key tile
  static constexpr int kVBytes = TK * D * 2;          // one value tile
  static constexpr int kPBytes = TQ * TK * 2;         // one P tile
  static constexpr int kQOff = 0;
  static constexpr int kKOff = 2 * kQBytes;
  static constexpr int kVOff = kKOff + 2 * kKBytes;
  static constexpr int kPOff = kVOff + 2 * kVBytes;
  static constexpr int kBarOff = kPOff + 4 * kPBytes;  // two P buffers per query tile
  static constexpr int kSmem = kBarOff + 256 + 1024;   // 225.25 KB for D = 64 (limit 227 KB)
  static constexpr int kOCol = 256;
  static constexpr int kPCol = kOCol + 2 * D;          // PT: P of tile t at columns kPCol + 64 t
  static_assert(kPCol + 2 * (TK / 2) <= 512, "TMEM columns");
};

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Packed f32x2 arithmetic (sm_100): two fp32 lanes in one 64-bit register pair per instruction.
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t pack2u(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ float lo_f(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo;
}
__device__ __forceinline__ float hi_f(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return hi;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// MN-major operand in the 128-byte swizzle layout: rows of 128 B along K (here: keys), the 64-element
// MN extent inside one row; SBO = 1024 B between 8-row groups along K.
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)(8192 >> 4) << 16;     // LBO: next 64-element MN block (unused for MN extent 64)
  d |= (uint64_t)(1024 >> 4) << 32;     // SBO
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kPFull / kPVFull: one barrier per (query tile t, P buffer b) at index 2 t + b; KV tile j uses
// buffer j & 1, so each of them completes once every second KV tile.
enum { kQFull = 0, kKFull = 1, kKEmpty = 3, kVFull = 5, kVEmpty = 7, kSFull = 9, kSFree = 11, kPFull = 13, kPVFull = 17,
       kNumBars = 21 };

// 320 threads: the compiler caps registers at 168 per thread (one CTA per SM); 200 does not launch.
// PT: P goes to tensor memory (64 columns per query tile) and P V reads its A operand from there,
// instead of P in shared memory (two buffers per tile) read through a descriptor.
template <int D, bool CAUSAL, bool VT, bool PT>
__global__ void __launch_bounds__(320, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O, float* __restrict__ lse2, int H,
                int S, float scale_log2) {
  using C = ACfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + C::kBarOff);
  uint32_t* tmem_slot = (uint32_t*)(bars + kNumBars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qblk = S / (2 * TQ);
  // causal: query-block-major order, every (batch, head)'s heaviest (last) query block dispatched
  // before any lighter one, so the last wave holds short CTAs.  Non-causal (equal CTAs): head-major
  // order, the query blocks of one (batch, head) in flight together, so its K and V are read from
  // HBM once and from L2 by the others.
  const int n_bh = (int)(gridDim.x / n_qblk);
  const int qi = CAUSAL ? (int)(blockIdx.x / n_bh) : (int)(blockIdx.x % n_qblk);
  const int qb = CAUSAL ? (n_qblk - 1 - qi) : qi;
  const int bh = CAUSAL ? (int)(blockIdx.x % n_bh) : (int)(blockIdx.x / n_qblk);
  const int q0 = qb * 2 * TQ;
  const int n_kv = CAUSAL ? (q0 + 2 * TQ) / TK : S / TK;
  const long long row_base = (long long)bh * S;  // row of (bh, 0) in the [B*H*S, D] views

  if (threadIdx.x == 0) {
    mbar_init(&bars[kQFull], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[kKFull + i], 1);
      mbar_init(&bars[kKEmpty + i], 1);
      mbar_init(&bars[kVFull + i], 1);
      mbar_init(&bars[kVEmpty + i], 1);
      mbar_init(&bars[kSFull + i], 1);
      mbar_init(&bars[kSFree + i], 128);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&bars[kPFull + i], 128);
      mbar_init(&bars[kPVFull + i], 1);
    }
    fence_barrier_init();
  }
  if (warp == 9) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  int* err = &g_tc_error_attn;

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(&bars[kQFull], 2 * C::kQBytes);
      tma_load_2d(&tmQ, &bars[kQFull], smem + C::kQOff, 0, (int)(row_base + q0));
      tma_load_2d(&tmQ, &bars[kQFull], smem + C::kQOff + C::kQBytes, 0, (int)(row_base + q0 + TQ));
      uint32_t kpar = 0, vpar = 0, kiss = 0, viss = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&bars[kKEmpty + st], ph ^ 1, kErrTimeoutEmpty, err)) break;
        mbar_arrive_expect_tx(&bars[kKFull + st], C::kKBytes);
        tma_load_2d(&tmK, &bars[kKFull + st], smem + C::kKOff + st * C::kKBytes, 0, (int)(row_base + j * TK));
        kiss |= 1u << st;
        kpar = (kpar & ~(1u << st)) | (ph << st);
        if (!mbar_wait(&bars[kVEmpty + st], ph ^ 1, kErrTimeoutEmpty, err)) break;
        mbar_arrive_expect_tx(&bars[kVFull + st], C::kVBytes);
        uint8_t* vdst = smem + C::kVOff + st * C::kVBytes;
        if (VT) {
          // V^T rows (bh*D + d), keys j*128 + [0,64) and + [64,128): two 64-key blocks of D rows
          tma_load_2d(&tmV, &bars[kVFull + st], vdst, j * TK, bh * D);
          tma_load_2d(&tmV, &bars[kVFull + st], vdst + D * 128, j * TK + 64, bh * D);
        } else {
          // V rows (keys) j*128 .. +128, the D = 64 values of a key in one 128-byte row
          tma_load_2d(&tmV, &bars[kVFull + st], vdst, 0, (int)(row_base + j * TK));
        }
        viss |= 1u << st;
        vpar = (vpar & ~(1u << st)) | (ph << st);
      }
      mbar_wait(&bars[kQFull], 0, kErrTimeoutOther, err);
      for (int s = 0; s < 2; ++s) {
        if (kiss & (1u << s)) mbar_wait(&bars[kKFull + s], (kpar >> s) & 1, kErrTimeoutOther, err);
        if (viss & (1u << s)) mbar_wait(&bars[kVFull + s], (vpar >> s) & 1, kErrTimeoutOther, err);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t id_s = idesc_f16(1, TQ, TK);
      const uint32_t id_pv = idesc_f16(1, TQ, D, !VT);
      const uint32_t q_addr = smem_u32(smem + C::kQOff);
      const uint32_t k_addr = smem_u32(smem + C::kKOff);
      const uint32_t v_addr = smem_u32(smem + C::kVOff);
      const uint32_t p_addr = smem_u32(smem + C::kPOff);
      auto issue_s = [&](int t, int j) {
        const int st = j & 1;
        const uint32_t qa = q_addr + t * C::kQBytes, ka = k_addr + st * C::kKBytes;
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          mma_f16_ss(tmem + t * 128, sw128_desc(qa + k * 32), sw128_desc(ka + k * 32), id_s, k != 0);
        mma_commit(&bars[kSFull + t]);
      };
      auto issue_pv = [&](int t, int j) {
        const int st = j & 1;
        const uint32_t pa = p_addr + (2 * t + (j & 1)) * C::kPBytes, va = v_addr + st * C::kVBytes;
#pragma unroll
        for (int k = 0; k < TK / 16; ++k) {
          const uint32_t off_p = (k / 4) * (TQ * 128) + (k % 4) * 32;
          const uint64_t bdesc = VT ? sw128_desc(va + (k / 4) * (D * 128) + (k % 4) * 32)
                                    : sw128_mn_desc(va + k * 16 * 128);
          mma_f16_ss(tmem + C::kOCol + t * D, sw128_desc(pa + off_p), bdesc, id_pv, (j | k) != 0);
        }
        mma_commit(&bars[kPVFull + 2 * t + (j & 1)]);
      };
      auto issue_pv_tmem = [&](int t, int j) {
        const uint32_t va = v_addr + (j & 1) * C::kVBytes;
#pragma unroll
        for (int k = 0; k < TK / 16; ++k) {
          const uint64_t bdesc = VT ? sw128_desc(va + (k / 4) * (D * 128) + (k % 4) * 32)
                                    : sw128_mn_desc(va + k * 16 * 128);
          // 16 keys of P = 8 columns (two bf16 per 32-bit column)
          mma_f16_ts(tmem + C::kOCol + t * D, tmem + C::kPCol + t * (TK / 2) + k * 8, bdesc, id_pv, (j | k) != 0);
        }
        mma_commit(&bars[kPVFull + 2 * t + (j & 1)]);
      };
      bool ok = mbar_wait(&bars[kQFull], 0, kErrTimeoutFull, err);
      if (ok) ok = mbar_wait(&bars[kKFull + 0], 0, kErrTimeoutFull, err);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        mma_commit(&bars[kKEmpty + 0]);
      }
      // Per KV tile j: both tiles' next scores S_t(j+1) as soon as their softmax has read S_t(j),
      // then both P V products.  A softmax group therefore never waits behind the other group's P,
      // and with two P buffers per tile it writes P(j+1) while P V(j) still reads P(j).
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const int ns = (j + 1) & 1;
        if (j + 1 < n_kv) {
          if (!mbar_wait(&bars[kKFull + ns], ((j + 1) >> 1) & 1, kErrTimeoutFull, err)) { ok = false; break; }
          for (int t = 0; t < 2 && ok; ++t) {
            if (!mbar_wait(&bars[kSFree + t], j & 1, kErrTimeoutFull, err)) { ok = false; break; }
            tc_fence_after();
            issue_s(t, j + 1);
          }
          if (!ok) break;
          mma_commit(&bars[kKEmpty + ns]);
        }
        if (!mbar_wait(&bars[kVFull + st], ph, kErrTimeoutFull, err)) { ok = false; break; }
        for (int t = 0; t < 2 && ok; ++t) {
          if (!mbar_wait(&bars[kPFull + 2 * t + (j & 1)], (j >> 1) & 1, kErrTimeoutFull, err)) { ok = false; break; }
          tc_fence_after();
          if (PT) issue_pv_tmem(t, j);
          else issue_pv(t, j);
        }
        if (!ok) break;
        mma_commit(&bars[kVEmpty + st]);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax warpgroups
    const int t = warp >> 2;                 // query tile 0 / 1
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;       // row inside the tile == TMEM lane
    const int qrow = q0 + t * TQ + r;        // query index inside the head
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_col = tmem + t * 128 + lane_off;
    const uint32_t o_col = tmem + C::kOCol + t * D + lane_off;
    uint8_t* const p_rows = smem + C::kPOff + 2 * t * C::kPBytes + r * 128;   // buffer b at + b * kPBytes
    float m_use = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!mbar_wait_warp(&bars[kSFull + t], j & 1, kErrTimeoutAcc, err)) { ok = false; break; }
      tc_fence_after();
      uint32_t sv[TK];
#pragma unroll
      for (int c = 0; c < TK; c += 16) tmem_ld16(s_col + c, *reinterpret_cast<uint32_t(*)[16]>(sv + c));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bars[kSFree + t]);        // S_t may be overwritten by the next Q K^T
      const int key0 = j * TK;
      if (CAUSAL && key0 + TK - 1 > q0 + t * TQ) {   // diagonal tile: keys after the query are -inf
#pragma unroll
        for (int e = 0; e < TK; ++e)
          if (key0 + e > qrow) sv[e] = 0xff800000u;
      }
      // row max of the raw scores (scale > 0 commutes with max): four independent chains of
      // three-way maxima, so consecutive instructions do not wait on each other
      float mc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) mc[i] = fmaxf(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1]));
#pragma unroll
      for (int e = 8; e < TK; e += 8)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          mc[i] = fmax3(mc[i], __uint_as_float(sv[e + 2 * i]), __uint_as_float(sv[e + 2 * i + 1]));
      float mx = fmax3(fmaxf(mc[0], mc[1]), mc[2], mc[3]);
      mx *= scale_log2;
      // The shared-memory form writes P buffer j & 1, last read by P V(j - 2); the tensor-memory form
      // has one P per tile, last read by P V(j - 1).  Wait for that product.
      uint8_t* const p_row = p_rows + (j & 1) * C::kPBytes;
      if (!PT && j >= 2 && !mbar_wait_warp(&bars[kPVFull + 2 * t + (j & 1)], ((j >> 1) - 1) & 1, kErrTimeoutAcc, err)) {
        ok = false;
        break;
      }
      if (PT && j >= 1 &&
          !mbar_wait_warp(&bars[kPVFull + 2 * t + ((j - 1) & 1)], ((j - 1) >> 1) & 1, kErrTimeoutAcc, err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // Lazy rescale.  The decision is per row, but tcgen05.ld / st are warp-collective
      // (.sync.aligned): the whole warp takes the TMEM path when any of its rows needs it, and rows
      // that do not rescale multiply by 1.  Rescaling O needs every earlier P V product done.
      const bool mine = mx > m_use + kRescaleThreshold;
      if (__any_sync(0xffffffffu, mine)) {
        const float m_new = mine ? mx : m_use;
        if (j > 0) {
          if (!mbar_wait_warp(&bars[kPVFull + 2 * t + ((j - 1) & 1)], ((j - 1) >> 1) & 1, kErrTimeoutAcc, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float f = mine ? ex2(m_use - m_new) : 1.f;
          l *= f;
#pragma unroll
          for (int c = 0; c < D; c += 16) {
            uint32_t v[16];
            tmem_ld16(o_col + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * f);
            tmem_st16(o_col + c, v);
          }
          tmem_wait_st();
        }
        m_use = m_new;
      }
      const float mu = m_use == -INFINITY ? 0.f : m_use;   // a row masked so far contributes p = 0
      // p = 2^(s * scale_log2 - m): one packed FMA per two scores, packed adds for the row sum
      const uint64_t sc2 = pack2(scale_log2, scale_log2), nm2 = pack2(-mu, -mu);
      uint64_t sum2[4] = {pack2(0.f, 0.f), pack2(0.f, 0.f), pack2(0.f, 0.f), pack2(0.f, 0.f)};   // independent sums
      const uint32_t p_col = tmem + C::kPCol + t * (TK / 2) + lane_off;
#pragma unroll
      for (int c = 0; c < TK; c += 32) {
        uint32_t pk[16];                     // keys c .. c+31, two bf16 per word
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const uint64_t x2 = ffma2(pack2u(sv[c + 2 * e], sv[c + 2 * e + 1]), sc2, nm2);
          const float p0 = ex2(lo_f(x2)), p1 = ex2(hi_f(x2));
          sum2[e & 3] = fadd2(sum2[e & 3], pack2(p0, p1));
          pk[e] = pack_bf16(p0, p1);
        }
        if (PT) {
          tmem_st16(p_col + c / 2, pk);      // 32 keys = 16 columns of this row's lane
        } else {
          // keys c .. c+31 = four 16-byte chunks of row r in the 64-key block c / 64 (128-byte swizzle)
          const int blk = c >> 6;
          const int ch0 = (c & 63) >> 3;
          uint8_t* rowp = p_row + blk * (TQ * 128);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *(uint4*)(rowp + (((ch0 + q) ^ (r & 7)) << 4)) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      const uint64_t s01 = fadd2(sum2[0], sum2[1]), s23 = fadd2(sum2[2], sum2[3]);
      const uint64_t stot = fadd2(s01, s23);
      l += lo_f(stot) + hi_f(stot);
      if (PT) tmem_wait_st();
      tc_fence_before();
      if (!PT) fence_async_smem();
      mbar_arrive(&bars[kPFull + 2 * t + (j & 1)]);
    }
    if (ok && mbar_wait_warp(&bars[kPVFull + 2 * t + ((n_kv - 1) & 1)], ((n_kv - 1) >> 1) & 1, kErrTimeoutAcc, err)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = O + (row_base + qrow) * D;
#pragma unroll
      for (int c = 0; c < D; c += 16) {
        uint32_t v[16];
        tmem_ld16(o_col + c, v);
        tmem_wait_ld();
        uint4 w0 = make_uint4(pack_bf16(__uint_as_float(v[0]) * inv, __uint_as_float(v[1]) * inv),
                              pack_bf16(__uint_as_float(v[2]) * inv, __uint_as_float(v[3]) * inv),
                              pack_bf16(__uint_as_float(v[4]) * inv, __uint_as_float(v[5]) * inv),
                              pack_bf16(__uint_as_float(v[6]) * inv, __uint_as_float(v[7]) * inv));
        uint4 w1 = make_uint4(pack_bf16(__uint_as_float(v[8]) * inv, __uint_as_float(v[9]) * inv),
                              pack_bf16(__uint_as_float(v[10]) * inv, __uint_as_float(v[11]) * inv),
                              pack_bf16(__uint_as_float(v[12]) * inv, __uint_as_float(v[13]) * inv),
                              pack_bf16(__uint_as_float(v[14]) * inv, __uint_as_float(v[15]) * inv));
        *(uint4*)(orow + c) = w0;
        *(uint4*)(orow + c + 8) = w1;
      }
      // log2-sum-exp of the scaled row (the backward recomputes P = 2^(s * scale_log2 - lse2))
      if (lse2) lse2[row_base + qrow] = l > 0.f ? (m_use == -INFINITY ? 0.f : m_use) + log2f(l) : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// V [BH, S, D] -> V^T [BH, D, S], 64 x 64 tiles through shared memory (VT variant only).
__global__ void __launch_bounds__(256) transpose_v_kernel(const uint16_t* __restrict__ v, uint16_t* __restrict__ vt, int S, int D) {
  __shared__ uint16_t tile[64][65];
  const int bh = blockIdx.z, s0 = blockIdx.x * 64, d0 = blockIdx.y * 64;
  const uint16_t* src = v + (long long)bh * S * D;
  uint16_t* dst = vt + (long long)bh * S * D;
  for (int i = threadIdx.x; i < 64 * 64; i += 256) {
    int rs = i / 64, cd = i % 64;
    tile[rs][cd] = src[(long long)(s0 + rs) * D + d0 + cd];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 64 * 64; i += 256) {
    int rd = i / 64, cs = i % 64;
    dst[(long long)(d0 + rd) * S + s0 + cs] = tile[cs][rd];
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace

EncodeTiledFn GetEncodeTiled();

static bool Map2D(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn enc = GetEncodeTiled();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, bool CAUSAL, bool VT, bool PT>
static int LaunchAttnP(const void* q, const void* k, const void* v, void* o, int B, int H, int S, float scale, cudaStream_t st,
                       float* lse2) {
  using Cf = ACfg<D>;
  static std::once_flag once[8];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 7], [] {
    cudaFuncSetAttribute(attn_fwd_kernel<D, CAUSAL, VT, PT>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::kSmem);
  });
  CUtensorMap mq, mk, mv;
  const uint64_t rows = (uint64_t)B * H * S;
  if (!Map2D(&mq, q, D, rows, 64, TQ) || !Map2D(&mk, k, D, rows, 64, TK)) return -2;
  if (VT) {
    if (!Map2D(&mv, v, (uint64_t)S, (uint64_t)B * H * D, 64, D)) return -2;
  } else {
    if (!Map2D(&mv, v, D, rows, 64, TK)) return -2;
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid((unsigned)(B * H * (S / (2 * TQ))));
  attn_fwd_kernel<D, CAUSAL, VT, PT><<<grid, 320, Cf::kSmem, st>>>(mq, mk, mv, (__nv_bfloat16*)o, lse2, H, S, scale_log2);
  CountLaunches();
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// P in tensor memory by default (measured 645 against 624 TFLOP/s at [4,16,4096,64]);
// B200_ATTN_P_SMEM=1 selects the shared-memory form as a cross-check.
template <int D, bool CAUSAL, bool VT>
static int LaunchAttn(const void* q, const void* k, const void* v, void* o, int B, int H, int S, float scale, cudaStream_t st,
                      float* lse2 = nullptr) {
  static const bool p_smem = std::getenv("B200_ATTN_P_SMEM") != nullptr && std::atoi(std::getenv("B200_ATTN_P_SMEM")) != 0;
  if (p_smem) return LaunchAttnP<D, CAUSAL, VT, false>(q, k, v, o, B, H, S, scale, st, lse2);
  return LaunchAttnP<D, CAUSAL, VT, true>(q, k, v, o, B, H, S, scale, st, lse2);
}

// B * H * S query rows must fit an int (grid and row arithmetic); the product is formed with
// overflow checks so that huge dimensions cannot wrap around to a small value.
bool AttentionShapeOk(int B, int H, int S, int D) {
  if (!(B > 0 && H > 0 && D == 64 && S > 0 && S % (2 * TQ) == 0)) return false;
  long long bh = 0, rows = 0;
  return !__builtin_mul_overflow((long long)B, (long long)H, &bh) && !__builtin_mul_overflow(bh, (long long)S, &rows) &&
         rows <= INT32_MAX;
}

// V read in place (MN-major operand); no scratch memory.
int AttentionFwd(const void* q, const void* k, const void* v, void* o, int B, int H, int S, int D, int causal, float scale,
                 cudaStream_t st) {
  if (!AttentionShapeOk(B, H, S, D)) return -1;
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o) % 16) return -1;
  if (causal) return LaunchAttn<64, true, false>(q, k, v, o, B, H, S, scale, st);
  return LaunchAttn<64, false, false>(q, k, v, o, B, H, S, scale, st);
}

// Training form: also writes lse2[B*H*S] (f32, log2 units of the scaled scores) for the backward.
int AttentionFwdLse(const void* q, const void* k, const void* v, void* o, float* lse2, int B, int H, int S, int D,
                    int causal, float scale, cudaStream_t st) {
  if (!AttentionShapeOk(B, H, S, D)) return -1;
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o | (uintptr_t)lse2) % 16) return -1;
  if (causal) return LaunchAttn<64, true, false>(q, k, v, o, B, H, S, scale, st, lse2);
  return LaunchAttn<64, false, false>(q, k, v, o, B, H, S, scale, st, lse2);
}

// Cross-check variant: V transposed into `vt` (B*H*S*D bf16 scratch) and read K-major.
int AttentionFwdWithVt(const void* q, const void* k, const void* v, void* vt, void* o, int B, int H, int S, int D,
                       int causal, float scale, cudaStream_t st) {
  if (!AttentionShapeOk(B, H, S, D) || (long long)B * H > 65535) return -1;   // B * H is the transpose's grid.z
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)vt | (uintptr_t)o) % 16) return -1;
  dim3 tg(S / 64, D / 64, B * H);
  transpose_v_kernel<<<tg, 256, 0, st>>>((const uint16_t*)v, (uint16_t*)vt, S, D);
  CountLaunches();
  if (causal) return LaunchAttn<64, true, true>(q, k, vt, o, B, H, S, scale, st);
  return LaunchAttn<64, false, true>(q, k, vt, o, B, H, S, scale, st);
}

int TakeAttnError() {
  int v = 0, z = 0;
  cudaMemcpyFromSymbol(&v, g_tc_error_attn, sizeof(int));
  if (v) cudaMemcpyToSymbol(g_tc_error_attn, &z, sizeof(int));
  return v;
}

}  // namespace b200k

extern "C" int b200_attention_fwd(const void* q, const void* k, const void* v, void* o, int B, int H, int S, int D,
                                  int causal, float scale, void* stream) {
  if (B == 0 || H == 0 || S == 0) return 0;
  return b200k::AttentionFwd(q, k, v, o, B, H, S, D, causal, scale, (cudaStream_t)stream);
}

extern "C" int b200_attention_fwd_lse(const void* q, const void* k, const void* v, void* o, float* lse2, int B, int H,
                                      int S, int D, int causal, float scale, void* stream) {
  if (B == 0 || H == 0 || S == 0) return 0;
  return b200k::AttentionFwdLse(q, k, v, o, lse2, B, H, S, D, causal, scale, (cudaStream_t)stream);
}

extern "C" int b200_attention_fwd_vt(const void* q, const void* k, const void* v, void* vt, void* o, int B, int H, int S,
                                     int D, int causal, float scale, void* stream) {
  if (B == 0 || H == 0 || S == 0) return 0;
  return b200k::AttentionFwdWithVt(q, k, v, vt, o, B, H, S, D, causal, scale, (cudaStream_t)stream);
}

// ------------------------------------------------------------------------------------------------
// Allocation-free variant of b200_attention_fwd_vt.  Its scratch (the transposed V) lives in this
// file-scope device array instead of memory the caller passes in.  The array is part of the
// library's device image: every GPU that loads this module holds it (32 MiB) until the process
// exits.  In host code `g_vt_noalloc_scratch` only names a host-side stand-in, so the device address
// is taken once per device with cudaGetSymbolAddress (with that device current) and cached.
namespace b200k {

constexpr size_t kNoAllocScratchBytes = 32u << 20;   // fits V^T for B*H*S*D <= 16 Mi bf16 elements

static __device__ __align__(256) unsigned char g_vt_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64];

// Device address of the scratch array for the current device; resolved on the first call per device.
static int NoAllocScratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -6;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_vt_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return -6;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

}  // namespace b200k

extern "C" int b200_attention_fwd_noalloc(const void* q, const void* k, const void* v, void* o, int B, int H, int S,
                                          int D, int causal, float scale, void* stream) {
  if (B == 0 || H == 0 || S == 0) return 0;
  if (!b200k::AttentionShapeOk(B, H, S, D)) return -1;   // bounds B * H * S before the size product
  const size_t need = (size_t)B * H * S * D * 2;
  if (need > b200k::kNoAllocScratchBytes) return -5;   // larger than the static scratch
  void* vt = nullptr;
  int rc = b200k::NoAllocScratch(&vt);
  if (rc != 0) return rc;
  return b200k::AttentionFwdWithVt(q, k, v, vt, o, B, H, S, D, causal, scale, (cudaStream_t)stream);
}
