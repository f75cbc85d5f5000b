// Per-tile arithmetic of the paged decode kernel: one compute warp, 16 keys
// of a 64-key K/V tile staged in shared memory by TMA (SWIZZLE_128B), all
// g = Hq/Hkv query heads of the kv group as the M = 16 rows of m16n8k16 MMAs.
#pragma once

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
// fp8 (e4m3) pool tiles.  The 64-row K and V code tiles (128 B rows,
// SWIZZLE_128B) are read straight from shared memory with 16-byte loads and
// widened in registers (cvt.rn.f16x2.e4m3x2: every e4m3 value is exact in
// f16), so both products run as f16 m16n8k16 MMAs with f32 accumulation:
//  * S = Q.codes^T: the reduction over D may visit D in any order as long as
//    Q's A fragments follow the same order, so k-step kk of lane (g, t) takes
//    D = 32t + 4kk + {0, 1} (b0) and + {2, 3} (b1): each lane reads 32
//    contiguous code bytes of its key row.  S is then scaled per key column
//    by that key's k-scale (fp32), which equals Q.(codes * k_scale) exactly.
//  * O += P'.codes_V with P' = P * v_scale(key) * 2^-E: the output column
//    order is free too (it is undone in the final combine), so d-tile dn,
//    column n is D = 16n + dn: each lane reads 16 contiguous bytes of the four
//    key rows of its B fragments and pairs them bytewise (prmt).  E is a
//    running power of two >= the largest v-scale seen (its f32 exponent
//    field), so P' stays in [0, 2) whatever the V magnitudes; O is kept in
//    units of 2^E and rescaled (exactly) when E grows.
// Q is converted to f16 once (exact for bf16 values within +-65504,
// saturated beyond).
// ---------------------------------------------------------------------------

// Four e4m3 codes (lowest byte first) -> two f16x2: codes {0,1} and {2,3}.
__device__ __forceinline__ void e4m3x4_to_h2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// two T values -> f16x2, saturated to the f16 range
template <typename T>
__device__ __forceinline__ uint32_t to_h2_sat(uint32_t u) {
  const float2 f = DT<T>::to_f2(u);
  return DT<__half>::from_f2(fminf(fmaxf(f.x, -65504.f), 65504.f),
                             fminf(fmaxf(f.y, -65504.f), 65504.f));
}

// f16 A fragments of the g query rows in the D order above.
template <typename T>
__device__ __forceinline__ void dec8_load_q(uint32_t (&qa)[8][4], const T* qrow, int g, int lane) {
  const int r0 = lane >> 2, r1 = r0 + 8, t = lane & 3;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int d = 32 * t + 4 * kk;
    const uint2 x0 = r0 < g ? *reinterpret_cast<const uint2*>(qrow + r0 * kDecD + d) : make_uint2(0, 0);
    const uint2 x1 = r1 < g ? *reinterpret_cast<const uint2*>(qrow + r1 * kDecD + d) : make_uint2(0, 0);
    qa[kk][0] = to_h2_sat<T>(x0.x);
    qa[kk][1] = to_h2_sat<T>(x1.x);
    qa[kk][2] = to_h2_sat<T>(x0.y);
    qa[kk][3] = to_h2_sat<T>(x1.y);
  }
}

// 2^(e - 127) from an f32 exponent field e (0 -> 0.0)
__device__ __forceinline__ float pow2_field(uint32_t e) { return __uint_as_float(e << 23); }

// This warp's 16 keys [wtok, wtok + 16) of the fp8 tile: kbase / vbase are
// the shared addresses of the K / V code tiles, ksc / vsc the tile's 64
// per-row scales; vexp is the warp's running exponent field E + 127.
template <bool kHi>
__device__ __forceinline__ void dec8_tile(const uint32_t (&qa)[8][4], DecState& st, uint32_t& vexp,
                                          uint32_t kbase, uint32_t vbase, const float* ksc,
                                          const float* vsc, int wtok, int valid, float scale_log2,
                                          int lane) {
  const int t = lane & 3, gq = lane >> 2;
  const int cq = 2 * t;
  float sc[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
    const uint32_t krow = (uint32_t)(wtok + nt * 8 + gq);
    const uint4 w0 = lds128(kbase + sw128_offset(krow, 2 * t));
    const uint4 w1 = lds128(kbase + sw128_offset(krow, 2 * t + 1));
    const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t b0, b1;
      e4m3x4_to_h2x2(w[kk], b0, b1);
      mma_16816<__half>(sc[nt], qa[kk], b0, b1);
    }
  }
  float vs[2][2];
  float mx0 = -INFINITY, mx1 = -INFINITY, vm = 0.f;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const float2 ks = *reinterpret_cast<const float2*>(ksc + wtok + nt * 8 + cq);
    const float2 v2 = *reinterpret_cast<const float2*>(vsc + wtok + nt * 8 + cq);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const bool ok = (nt * 8 + cq + e) < valid;
      const float f = (e ? ks.y : ks.x) * scale_log2;
      vs[nt][e] = ok ? (e ? v2.y : v2.x) : 0.f;
      vm = fmaxf(vm, vs[nt][e]);
      sc[nt][e] = ok ? sc[nt][e] * f : -INFINITY;
      mx0 = fmaxf(mx0, sc[nt][e]);
      if (kHi) {
        sc[nt][e + 2] = ok ? sc[nt][e + 2] * f : -INFINITY;
        mx1 = fmaxf(mx1, sc[nt][e + 2]);
      }
    }
  }
  // the 16 keys' largest v-scale (lanes of a quad hold all of them)
  vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, 1));
  vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, 2));
  const uint32_t vnew = max(vexp, min(254u, __float_as_uint(vm) >> 23));  // inf/NaN: clamp
  const float vfac = vnew == vexp ? 1.f
                     : (int)(vnew - vexp) < 127 ? pow2_field(127u - (vnew - vexp)) : 0.f;
  vexp = vnew;
  const float vinv = pow2_field(254u - vnew);  // 2^-E

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
  const float f0 = al0 * vfac, f1 = al1 * vfac;
  if (f0 != 1.f || f1 != 1.f) {
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      st.o[n][0] *= f0;
      st.o[n][1] *= f0;
      if (kHi) {
        st.o[n][2] *= f1;
        st.o[n][3] *= f1;
      }
    }
  }
  uint32_t pa[4];
  const float w00 = vs[0][0] * vinv, w01 = vs[0][1] * vinv;
  const float w10 = vs[1][0] * vinv, w11 = vs[1][1] * vinv;
  pa[0] = DT<__half>::from_f2(sc[0][0] * w00, sc[0][1] * w01);
  pa[1] = kHi ? DT<__half>::from_f2(sc[0][2] * w00, sc[0][3] * w01) : 0u;
  pa[2] = DT<__half>::from_f2(sc[1][0] * w10, sc[1][1] * w11);
  pa[3] = kHi ? DT<__half>::from_f2(sc[1][2] * w10, sc[1][3] * w11) : 0u;
  // B fragment keys of this lane: wtok + cq + {0,1} (b0), + 8 + {0,1} (b1);
  // missing keys' codes (stale rows, possibly NaN codes) are zeroed
  const uint32_t keep_lo = (cq < valid ? 0x0000ffffu : 0u) | (cq + 1 < valid ? 0xffff0000u : 0u);
  const uint32_t keep_hi =
      (cq + 8 < valid ? 0x0000ffffu : 0u) | (cq + 9 < valid ? 0xffff0000u : 0u);
  const uint32_t ra = (uint32_t)(wtok + cq), rb = ra + 8;
  const uint4 A0 = lds128(vbase + sw128_offset(ra, gq));
  const uint4 A1 = lds128(vbase + sw128_offset(ra + 1, gq));
  const uint4 B0 = lds128(vbase + sw128_offset(rb, gq));
  const uint4 B1 = lds128(vbase + sw128_offset(rb + 1, gq));
  const uint32_t a0[4] = {A0.x, A0.y, A0.z, A0.w}, a1[4] = {A1.x, A1.y, A1.z, A1.w};
  const uint32_t c0[4] = {B0.x, B0.y, B0.z, B0.w}, c1[4] = {B1.x, B1.y, B1.z, B1.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // bytes 4i .. 4i + 3 of each row: d-tiles dn = 4i .. 4i + 3
    uint32_t l0, l1, l2, l3, h0, h1, h2, h3;
    e4m3x4_to_h2x2(__byte_perm(a0[i], a1[i], 0x5140), l0, l1);
    e4m3x4_to_h2x2(__byte_perm(a0[i], a1[i], 0x7362), l2, l3);
    e4m3x4_to_h2x2(__byte_perm(c0[i], c1[i], 0x5140), h0, h1);
    e4m3x4_to_h2x2(__byte_perm(c0[i], c1[i], 0x7362), h2, h3);
    mma_16816<__half>(st.o[4 * i + 0], pa, l0 & keep_lo, h0 & keep_hi);
    mma_16816<__half>(st.o[4 * i + 1], pa, l1 & keep_lo, h1 & keep_hi);
    mma_16816<__half>(st.o[4 * i + 2], pa, l2 & keep_lo, h2 & keep_hi);
    mma_16816<__half>(st.o[4 * i + 3], pa, l3 & keep_lo, h3 & keep_hi);
  }
}

// TMA row of key tile j0 of sequence b: through the page table (pages of
// page_size rows; an out-of-range page id is recorded and read as page 0 so
// the waiting consumers still get their bytes) or contiguous from cu_k[b].
__device__ __forceinline__ int64_t dec_tile_row(const uint32_t* block_tables, int64_t bt_stride,
                                                int64_t num_blocks, int page_size,
                                                const uint32_t* cu_k, int b, int j0, int* err) {
  if (block_tables) {
    uint32_t page = block_tables[(int64_t)b * bt_stride + j0 / page_size];
    if ((int64_t)page >= num_blocks) {
      record_error(err, NVKV_DEVERR_BLOCK_RANGE);
      page = 0;
    }
    return (int64_t)page * page_size + (j0 % page_size);
  }
  return (int64_t)cu_k[b] + j0;
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
