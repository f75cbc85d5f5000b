// Per-tile arithmetic of the paged decode kernel: one compute warp, 16 keys
// of a 64-key K/V tile staged in shared memory by TMA (SWIZZLE_128B), all
// g = Hq/Hkv query heads of the kv group as the M = 16 rows of m16n8k16 MMAs.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace nvkv {

constexpr int kDecD = 128;
constexpr int kDecTile = 64;
constexpr int kDecStages = 3;
constexpr int kDecComputeWarps = 4;
constexpr int kDecThreads = (kDecComputeWarps + 1) * 32;
constexpr int kDecHalfBytes = kDecTile * 128;      // 64 rows x 64 elems x 2 B
constexpr int kDecTileBytes = 2 * kDecHalfBytes;   // one K (or V) tile
constexpr int kDecStageBytes = 2 * kDecTileBytes;  // K + V
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ uint32_t ld_u32(const void* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

// A fragments of the g query rows (rows >= g are zero), D = 128 as 8 k-steps.
template <typename T>
__device__ __forceinline__ void dec_load_q(uint32_t (&qa)[8][4], const T* qrow, int g, int lane) {
  const int r0 = lane >> 2, r1 = r0 + 8;
  const int cq = (lane & 3) * 2;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int d = kk * 16 + cq;
    qa[kk][0] = r0 < g ? ld_u32(qrow + r0 * kDecD + d) : 0u;
    qa[kk][1] = r1 < g ? ld_u32(qrow + r1 * kDecD + d) : 0u;
    qa[kk][2] = r0 < g ? ld_u32(qrow + r0 * kDecD + d + 8) : 0u;
    qa[kk][3] = r1 < g ? ld_u32(qrow + r1 * kDecD + d + 8) : 0u;
  }
}

// Online-softmax state of one warp: O rows r0 = lane/4 and r1 = r0 + 8.
struct DecState {
  float o[16][4];
  float m0, m1, l0, l1;
  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
  }
};

// This warp's 16 keys [wtok, wtok + 16) of the tile at kbase / vbase (shared
// addresses); `valid` = how many of them exist (<= 0: nothing to do).
// S = Q.K^T (two n8 key tiles), fp32 online softmax with quad shuffles, then
// O += P.V with P re-packed from the S accumulators as the A operand and
// the V fragments of missing keys zeroed (stale cache rows never reach O).
// kHi = false (group size <= 8): rows 8..15 (r1) are padding, so their
// softmax is skipped and their P rows are zero -- half of the exp2 and
// conversion work (the XU pipe) -- while the MMAs stay as they are.
template <typename T, bool kHi>
__device__ __forceinline__ void dec_tile(const uint32_t (&qa)[8][4], DecState& st, uint32_t kbase,
                                         uint32_t vbase, int wtok, int valid, float scale_log2,
                                         int lane) {
  const int cq = (lane & 3) * 2;
  const int lrow = lane & 7;   // row inside an 8x8 ldmatrix tile
  const int lmat = lane >> 3;  // which of the four 8x8 tiles this lane addresses
  float sc[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
    const uint32_t krow = (uint32_t)(wtok + nt * 8 + lrow);
#pragma unroll
    for (int kk = 0; kk < 8; kk += 2) {
      const uint32_t chunk = (uint32_t)(2 * kk + lmat);  // 16-byte chunk along D (0..15)
      const uint32_t addr = kbase + (chunk >> 3) * kDecHalfBytes + sw128_offset(krow, chunk & 7);
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4(b0, b1, b2, b3, addr);
      mma_16816<T>(sc[nt], qa[kk], b0, b1);
      mma_16816<T>(sc[nt], qa[kk + 1], b2, b3);
    }
  }
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const bool ok = (nt * 8 + cq + e) < valid;
      sc[nt][e] = ok ? sc[nt][e] * scale_log2 : -INFINITY;
      mx0 = fmaxf(mx0, sc[nt][e]);
      if (kHi) {
        sc[nt][e + 2] = ok ? sc[nt][e + 2] * scale_log2 : -INFINITY;
        mx1 = fmaxf(mx1, sc[nt][e + 2]);
      }
    }
  }
  mx0 = warp_max_xor(warp_max_xor(mx0, 1), 2);
  const float mn0 = fmaxf(st.m0, mx0);
  const float mu0 = mn0 == -INFINITY ? 0.f : mn0;
  const float al0 = exp2f(st.m0 - mu0);
  st.m0 = mn0;
  float al1 = 1.f;
  if (kHi) {
    mx1 = warp_max_xor(warp_max_xor(mx1, 1), 2);
    const float mn1 = fmaxf(st.m1, mx1);
    const float mu1 = mn1 == -INFINITY ? 0.f : mn1;
    al1 = exp2f(st.m1 - mu1);
    st.m1 = mn1;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      sc[nt][2] = exp2f(sc[nt][2] - mu1);
      sc[nt][3] = exp2f(sc[nt][3] - mu1);
    }
    st.l1 = st.l1 * al1 + (sc[0][2] + sc[0][3] + sc[1][2] + sc[1][3]);
  }
  float ps0 = 0.f;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      sc[nt][e] = exp2f(sc[nt][e] - mu0);
      ps0 += sc[nt][e];
    }
  }
  st.l0 = st.l0 * al0 + ps0;
  if (al0 != 1.f || al1 != 1.f) {
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      st.o[n][0] *= al0;
      st.o[n][1] *= al0;
      if (kHi) {
        st.o[n][2] *= al1;
        st.o[n][3] *= al1;
      }
    }
  }
  uint32_t pa[4];
  pa[0] = DT<T>::from_f2(sc[0][0], sc[0][1]);
  pa[1] = kHi ? DT<T>::from_f2(sc[0][2], sc[0][3]) : 0u;
  pa[2] = DT<T>::from_f2(sc[1][0], sc[1][1]);
  pa[3] = kHi ? DT<T>::from_f2(sc[1][2], sc[1][3]) : 0u;
  // keys this lane's B fragments carry: wtok + cq + {0,1} (b0), + 8 (b1)
  const uint32_t keep_lo = (cq < valid ? 0x0000ffffu : 0u) | (cq + 1 < valid ? 0xffff0000u : 0u);
  const uint32_t keep_hi =
      (cq + 8 < valid ? 0x0000ffffu : 0u) | (cq + 9 < valid ? 0xffff0000u : 0u);
  const uint32_t vrow = (uint32_t)(wtok + (lmat & 1) * 8 + lrow);
#pragma unroll
  for (int dn = 0; dn < 16; dn += 2) {
    const uint32_t chunk = (uint32_t)(dn + (lmat >> 1));
    const uint32_t addr = vbase + (chunk >> 3) * kDecHalfBytes + sw128_offset(vrow, chunk & 7);
    uint32_t b0, b1, b2, b3;
    ldmatrix_x4_trans(b0, b1, b2, b3, addr);
    b0 &= keep_lo;
    b1 &= keep_hi;
    b2 &= keep_lo;
    b3 &= keep_hi;
    mma_16816<T>(st.o[dn], pa, b0, b1);
    mma_16816<T>(st.o[dn + 1], pa, b2, b3);
  }
}

// ---------------------------------------------------------------------------
// fp8 (e4m3) pool tiles, transposed products.  The K and V code tiles (64
// rows of 128 B, SWIZZLE_128B) are read straight from shared memory with
// 16-byte loads.  Keys and D take the M side of the MMAs and the query heads
// of the group the N side (8 per n-tile, kNt = 1 for groups of <= 8 heads,
// 2 for <= 16), so no M rows are padding:
//  * S^T = codes_K . Q^T on m16n8k32 e4m3 MMAs.  A = the K code rows as they
//    sit in shared memory: lane (g, t) reads 32 contiguous bytes of key rows
//    g and g + 8 of its warp's 16 keys, and k-step kk covers D = 32t + 8kk +
//    {0..3} (a0, a1) and + {4..7} (a2, a3) -- a reduction may visit D in any
//    order as long as both operands follow it.  B = Q as a sum of e4m3 pieces
//    (Dec8Q) in the same D order.  Each S^T row is then scaled by its key's
//    k-scale, which equals Q.(codes * k_scale) exactly.
//  * O^T += codes_V^T . P'^T on m16n8k16 f16 MMAs.  The order of O's D rows is
//    free too (the final combine undoes it): m-tile mt, row m is D = 16(m mod
//    8) + 8(m / 8) + mt, so lane (g, t) reads 16 contiguous bytes at D = 16g
//    of key rows 2t, 2t + 1, 2t + 8, 2t + 9, pairs them bytewise (prmt) and
//    widens them with cvt.rn.f16x2.e4m3x2 (every e4m3 value is exact in f16).
//    P' = P * v_scale(key) * 2^-E, E a running power of two >= the largest
//    v-scale seen (its f32 exponent field vexp), so P' < 2 whatever the V
//    magnitudes; O is kept in units of 2^E and rescaled exactly when E grows.
//    The S^T fragment holds P' per (key row, head pair); four shuffles per
//    n-tile bring each lane the (key pair, head) entries of its B fragments.
// ---------------------------------------------------------------------------

// Four e4m3 codes (lowest byte first) -> two f16x2: codes {0,1} and {2,3}.
__device__ __forceinline__ void e4m3x4_to_h2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

// e4m3 codes of (a, b), low byte = a (nearest even, saturating at 448)
__device__ __forceinline__ uint32_t e4m3x2_pack(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return r;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// D = A.B + C, m16n8k32, A and B e4m3, f32 accumulate.
__device__ __forceinline__ void mma_e4m3_16832(float (&c)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 2^(e - 127) from an f32 exponent field e (0 -> 0.0)
__device__ __forceinline__ float pow2_field(uint32_t e) { return __uint_as_float(e << 23); }

// Q as a sum of e4m3 pieces: Q * 2^sq = q_0 + q_1 (+ q_2), each piece the
// e4m3 rounding of what the pieces before it left over.  sq puts the group's
// largest |Q| just below 256, so two pieces hold a bf16 value exactly (8
// significant bits: the first piece's rounding error is an integer multiple
// of the value's ulp of at most 8 ulps) as long as |Q * 2^sq| >= 1/4, and
// three pieces an f16 value; smaller elements keep at least 4 bits.
template <typename T>
struct Dec8Q {
  static constexpr int kPieces = std::is_same<T, __half>::value ? 3 : 2;
};

// Lane (g, t) of n-tile j holds head 8j + g, D = 32t .. 32t + 31 of every
// piece: qb[piece][j][w] = the codes of D = 32t + 4w .. 32t + 4w + 3.  Heads
// >= g (the group size) are zero.  Returns 2^-sq.
template <typename T, int kP, int kNt>
__device__ __forceinline__ float dec8_load_q(uint32_t (&qb)[kP][kNt][8], const T* qrow, int g,
                                             int lane) {
  const int gq = lane >> 2, t = lane & 3;
  float x[kNt][32];
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < kNt; ++j) {
    const int h = 8 * j + gq;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 u = h < g ? *reinterpret_cast<const uint4*>(qrow + h * kDecD + 32 * t + 8 * c)
                            : make_uint4(0, 0, 0, 0);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = DT<T>::to_f2(w[k]);
        x[j][8 * c + 2 * k] = f.x;
        x[j][8 * c + 2 * k + 1] = f.y;
        m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  // m * 2^sq < 256 <= 448 with sq = 7 - floor(log2 m)
  const int e = (int)((__float_as_uint(m) >> 23) & 0xFFu);  // biased exponent of m
  const int sq = m > 0.f ? min(127, 134 - e) : 0;
  const float up = __uint_as_float((uint32_t)(127 + sq) << 23);
#pragma unroll
  for (int j = 0; j < kNt; ++j)
#pragma unroll
    for (int i = 0; i < 32; ++i) x[j][i] *= up;
#pragma unroll
  for (int pc = 0; pc < kP; ++pc) {
#pragma unroll
    for (int j = 0; j < kNt; ++j) {
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        float* v = &x[j][4 * w];
        const uint32_t wd = e4m3x2_pack(v[0], v[1]) | (e4m3x2_pack(v[2], v[3]) << 16);
        qb[pc][j][w] = wd;
        if (pc + 1 < kP) {  // what this piece leaves over
          uint32_t lo, hi;
          e4m3x4_to_h2x2(wd, lo, hi);
          const float2 a = DT<__half>::to_f2(lo), b = DT<__half>::to_f2(hi);
          v[0] -= a.x;
          v[1] -= a.y;
          v[2] -= b.x;
          v[3] -= b.y;
        }
      }
    }
  }
  return __uint_as_float((uint32_t)(127 - sq) << 23);
}

// Online-softmax state of one warp, transposed: lane (g, t) holds, per n-tile
// j, heads 8j + 2t + {0, 1}: their running max m (the same on every g), its
// partial row sum l over the keys it saw, and O^T rows D = 16g + mt (o[..][0
// / 1]) and 16g + 8 + mt (o[..][2 / 3]).
template <int kNt>
struct Dec8State {
  float o[kNt][8][4];
  float m[kNt][2], l[kNt][2];
  uint32_t vexp;  // O in units of 2^(vexp - 127)
  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int j = 0; j < kNt; ++j) {
#pragma unroll
      for (int n = 0; n < 8; ++n) o[j][n][0] = o[j][n][1] = o[j][n][2] = o[j][n][3] = 0.f;
      m[j][0] = m[j][1] = -INFINITY;
      l[j][0] = l[j][1] = 0.f;
    }
    vexp = 0;
  }
};

__device__ __forceinline__ float dec_ex2(float x) {  // 2^x on MUFU (-inf -> 0)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// This warp's 32 keys [wtok, wtok + 32) of the fp8 tile, as two 16-key
// halves u = 0, 1 (keys wtok + 16u + 0..15) that share one online-softmax
// update: kbase / vbase are the shared addresses of the K / V code tiles,
// ksc / vsc the tile's 64 row scales.  kPart: fewer than 32 of the keys
// exist (`valid`), so the missing ones are masked (their codes may be stale
// or NaN); otherwise nothing is.
template <int kP, int kNt, bool kPart>
__device__ __forceinline__ void dec8_tile(const uint32_t (&qb)[kP][kNt][8], Dec8State<kNt>& st,
                                          uint32_t kbase, uint32_t vbase, const float* ksc,
                                          const float* vsc, int wtok, int valid, float scale_log2,
                                          int lane) {
  const int t = lane & 3, gq = lane >> 2;
  // ---- S^T: key rows 16u + gq (x = 0) and 16u + gq + 8 (x = 1) ----
  float s[2][kNt][4];  // [u][j][c]: c = 2x + e, head 8j + 2t + e
  {
    // rows r and r + 8k share r's swizzle phase: one offset per chunk
    const uint32_t k0 = kbase + sw128_offset((uint32_t)(wtok + gq), 2 * t);
    const uint32_t k1 = kbase + sw128_offset((uint32_t)(wtok + gq), 2 * t + 1);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint4 a0 = lds128(k0 + u * 2048), a1 = lds128(k1 + u * 2048);
      const uint4 b0 = lds128(k0 + u * 2048 + 1024), b1 = lds128(k1 + u * 2048 + 1024);
      const uint32_t ka[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const uint32_t kb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      float acc[kNt][kP][4];  // one chain per (n-tile, piece): four MMAs deep
#pragma unroll
      for (int j = 0; j < kNt; ++j)
#pragma unroll
        for (int pc = 0; pc < kP; ++pc) {
          acc[j][pc][0] = acc[j][pc][1] = acc[j][pc][2] = acc[j][pc][3] = 0.f;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_e4m3_16832(acc[j][pc], ka[2 * kk], kb[2 * kk], ka[2 * kk + 1], kb[2 * kk + 1],
                           qb[pc][j][2 * kk], qb[pc][j][2 * kk + 1]);
        }
#pragma unroll
      for (int j = 0; j < kNt; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v = acc[j][0][c];
#pragma unroll
          for (int pc = 1; pc < kP; ++pc) v += acc[j][pc][c];
          s[u][j][c] = v;
        }
    }
  }
  // the lane's four keys 16u + 8x + gq: scales, presence
  float f[2][2], w[2][2];
  bool ok[2][2];
  float vm = 0.f;
#pragma unroll
  for (int u = 0; u < 2; ++u)
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      const int k = 16 * u + 8 * x + gq;
      ok[u][x] = !kPart || k < valid;
      f[u][x] = ksc[wtok + k] * scale_log2;
      w[u][x] = ok[u][x] ? vsc[wtok + k] : 0.f;
      vm = fmaxf(vm, w[u][x]);
    }
  // the 32 keys' largest v-scale
  vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, 4));
  vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, 8));
  vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, 16));
  const uint32_t vnew = max(st.vexp, min(254u, __float_as_uint(vm) >> 23));  // inf/NaN: clamp
  const float vfac = vnew == st.vexp ? 1.f
                     : (int)(vnew - st.vexp) < 127 ? pow2_field(127u - (vnew - st.vexp)) : 0.f;
  st.vexp = vnew;
  const float vinv = pow2_field(254u - vnew);  // 2^-E
#pragma unroll
  for (int u = 0; u < 2; ++u)
#pragma unroll
    for (int x = 0; x < 2; ++x) w[u][x] *= vinv;

  uint32_t xp[2][2][kNt];  // P' of key 16u + 8x + gq, heads 8j + 2t + {0, 1}
#pragma unroll
  for (int j = 0; j < kNt; ++j) {
    float fac[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float sv[2][2];
      float mx = -INFINITY;
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          sv[u][x] = ok[u][x] ? s[u][j][2 * x + e] * f[u][x] : -INFINITY;
          mx = fmaxf(mx, sv[u][x]);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float mn = fmaxf(st.m[j][e], mx);
      const float mu = mn == -INFINITY ? 0.f : mn;
      const float al = dec_ex2(st.m[j][e] - mu);
      st.m[j][e] = mn;
      float ps = 0.f;
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const float pv = dec_ex2(sv[u][x] - mu);
          ps += pv;
          s[u][j][2 * x + e] = pv * w[u][x];
        }
      st.l[j][e] = st.l[j][e] * al + ps;
      fac[e] = al * vfac;
    }
    if (fac[0] != 1.f || fac[1] != 1.f) {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        st.o[j][n][0] *= fac[0];
        st.o[j][n][1] *= fac[1];
        st.o[j][n][2] *= fac[0];
        st.o[j][n][3] *= fac[1];
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int x = 0; x < 2; ++x)
        xp[u][x][j] = DT<__half>::from_f2(s[u][j][2 * x], s[u][j][2 * x + 1]);
  }
  // ---- O^T += V^T . P'^T, per half ----
  // B fragments of n-tile j: b0 = P'[keys 2t, 2t + 1][head 8j + gq], b1 = the
  // same for keys 2t + 8, 2t + 9 (of the half).  Key k's pair of heads
  // (gq & ~1, gq | 1) sits in lane 4 (k mod 8) + gq / 2, in xp[u][k / 8].
  const int src0 = 4 * (2 * t) + (gq >> 1), src1 = src0 + 4;
  const uint32_t sel = (gq & 1) ? 0x7632u : 0x5410u;
  const int cq = 2 * t;
  const uint32_t v0 = vbase + sw128_offset((uint32_t)(wtok + cq), gq);
  const uint32_t v1 = vbase + sw128_offset((uint32_t)(wtok + cq + 1), gq);
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    uint32_t pb0[kNt], pb1[kNt];
#pragma unroll
    for (int j = 0; j < kNt; ++j) {
      const uint32_t a0 = __shfl_sync(0xffffffffu, xp[u][0][j], src0);
      const uint32_t a1 = __shfl_sync(0xffffffffu, xp[u][0][j], src1);
      const uint32_t b0 = __shfl_sync(0xffffffffu, xp[u][1][j], src0);
      const uint32_t b1 = __shfl_sync(0xffffffffu, xp[u][1][j], src1);
      pb0[j] = __byte_perm(a0, a1, sel);
      pb1[j] = __byte_perm(b0, b1, sel);
    }
    const int vk = valid - 16 * u;  // keys of this half that exist
    const uint32_t keep_lo =
        !kPart ? ~0u : (cq < vk ? 0x0000ffffu : 0u) | (cq + 1 < vk ? 0xffff0000u : 0u);
    const uint32_t keep_hi =
        !kPart ? ~0u : (cq + 8 < vk ? 0x0000ffffu : 0u) | (cq + 9 < vk ? 0xffff0000u : 0u);
    // rows 16u + cq (+1) and + 8: the same swizzle phase as rows cq (+1)
    const uint4 A0 = lds128(v0 + u * 2048), A1 = lds128(v1 + u * 2048);
    const uint4 B0 = lds128(v0 + u * 2048 + 1024), B1 = lds128(v1 + u * 2048 + 1024);
    const uint32_t x0[4] = {A0.x, A0.y, A0.z, A0.w}, x1[4] = {A1.x, A1.y, A1.z, A1.w};
    const uint32_t y0[4] = {B0.x, B0.y, B0.z, B0.w}, y1[4] = {B1.x, B1.y, B1.z, B1.w};
#pragma unroll
    for (int i = 0; i < 2; ++i) {  // bytes 4i .. 4i + 3 (rows m < 8) and 8 + 4i .. (m >= 8)
      uint32_t a[4][4];            // [mt - 4i][a0..a3]
      e4m3x4_to_h2x2(__byte_perm(x0[i], x1[i], 0x5140), a[0][0], a[1][0]);
      e4m3x4_to_h2x2(__byte_perm(x0[i], x1[i], 0x7362), a[2][0], a[3][0]);
      e4m3x4_to_h2x2(__byte_perm(x0[i + 2], x1[i + 2], 0x5140), a[0][1], a[1][1]);
      e4m3x4_to_h2x2(__byte_perm(x0[i + 2], x1[i + 2], 0x7362), a[2][1], a[3][1]);
      e4m3x4_to_h2x2(__byte_perm(y0[i], y1[i], 0x5140), a[0][2], a[1][2]);
      e4m3x4_to_h2x2(__byte_perm(y0[i], y1[i], 0x7362), a[2][2], a[3][2]);
      e4m3x4_to_h2x2(__byte_perm(y0[i + 2], y1[i + 2], 0x5140), a[0][3], a[1][3]);
      e4m3x4_to_h2x2(__byte_perm(y0[i + 2], y1[i + 2], 0x7362), a[2][3], a[3][3]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t af[4] = {a[q][0] & keep_lo, a[q][1] & keep_lo, a[q][2] & keep_hi,
                                a[q][3] & keep_hi};
#pragma unroll
        for (int j = 0; j < kNt; ++j) mma_16816<__half>(st.o[j][4 * i + q], af, pb0[j], pb1[j]);
      }
    }
  }
}

// Column of D = d of head h in the fp8 path's final-combine buffer: the low
// five bits are XOR-ed with (d / 32 mod 4, h / 2 mod 4), so a warp's scatter
// of its O^T fragments and the row-wise reads both hit 32 distinct banks.
__device__ __forceinline__ int dec8_ofin_col(int d, int h) {
  return (d & ~31) | ((d & 31) ^ (((d >> 5) & 3) | (((h >> 1) & 3) << 2)));
}

// The warp's (m, l) per head into red ([warp][m | l][16]) and its O rows,
// times `f`(head) * 2^E, into ow ([16 heads][128], dec8_ofin_col order).
template <int kNt>
__device__ __forceinline__ void dec8_put_ml(Dec8State<kNt>& st, float* red, int warp, int lane) {
  const int t = lane & 3, gq = lane >> 2;
#pragma unroll
  for (int j = 0; j < kNt; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float l = st.l[j][e];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      st.l[j][e] = l;
      if (gq == 0) {
        const int h = 8 * j + 2 * t + e;
        red[(warp * 2 + 0) * 16 + h] = st.m[j][e];
        red[(warp * 2 + 1) * 16 + h] = l;
      }
    }
}

template <int kNt>
__device__ __forceinline__ void dec8_put_o(const Dec8State<kNt>& st, const float* red,
                                           float* ow, int nwarps, int lane) {
  const int t = lane & 3, gq = lane >> 2;
  const float p2 = pow2_field(st.vexp);
#pragma unroll
  for (int j = 0; j < kNt; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int h = 8 * j + 2 * t + e;
      float ms = -INFINITY;
      for (int w = 0; w < nwarps; ++w) ms = fmaxf(ms, red[(w * 2) * 16 + h]);
      const float f = exp2f(st.m[j][e] - (ms == -INFINITY ? 0.f : ms)) * p2;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int d0 = 16 * gq + n, d1 = d0 + 8;
        ow[h * kDecD + dec8_ofin_col(d0, h)] = st.o[j][n][e] * f;
        ow[h * kDecD + dec8_ofin_col(d1, h)] = st.o[j][n][e + 2] * f;
      }
    }
}

// Four TMA loads of one stage: K and V, the two 64-element halves of D.
__device__ __forceinline__ void dec_load_stage(uint8_t* st, uint64_t* full, const CUtensorMap* mk,
                                               const CUtensorMap* mv, int kvh, int64_t row) {
  mbar_arrive_expect_tx(full, kDecStageBytes);
  tma_load_3d(st, mk, full, 0, kvh, (int)row);
  tma_load_3d(st + kDecHalfBytes, mk, full, 64, kvh, (int)row);
  tma_load_3d(st + kDecTileBytes, mv, full, 0, kvh, (int)row);
  tma_load_3d(st + kDecTileBytes + kDecHalfBytes, mv, full, 64, kvh, (int)row);
}

}  // namespace nvkv
