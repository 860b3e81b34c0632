// Shared compile-time structure of the path-preserving ICTC tensor product.
//
// The path list is the triangle/parity-allowed (l1, l2, l3) with l1 <= LI,
// l2 <= LE, l3 <= LO, enumerated l1 outermost, l2, then l3 (the operator
// factory order of ictc_o3/operators.py:54-55 filtered through
// ictc_o3/basis/ictd_irreps.py:2159-2172).  Since groups are sorted by
// (l1, l2) (ictd_irreps.py:2194-2211) the group order equals the path order,
// so a path's output block is at (sum_{l<l3} count_l (2l+1) + offset_p (2l3+1))
// angular rows of C channels (ictd_irreps.py:2512-2533, operators.py:107-115).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <utility>

namespace ictc {

constexpr int kMaxPaths = 64;

enum Layout : int { kIrMul = 0, kMulIr = 1 };

struct PathTable {
  int np = 0;
  int l1[kMaxPaths] = {};
  int l2[kMaxPaths] = {};
  int l3[kMaxPaths] = {};
  int bond_off[kMaxPaths] = {};  // first bond column of the path: sum m1*m3
  int coef_off[kMaxPaths] = {};  // first dense CG value: sum m1*m2*m3
  int out_row[kMaxPaths] = {};   // first angular output row of the path block
  int bond_width = 0;
  int coef_total = 0;
  int out_rows = 0;              // output width / C
};

constexpr int cmax(int a, int b) { return a > b ? a : b; }
constexpr int cabs(int a) { return a < 0 ? -a : a; }

constexpr PathTable make_paths(int LI, int LE, int LO) {
  PathTable t{};
  int lmax = cmax(LI, cmax(LE, LO));
  for (int i = 0; i <= lmax; ++i)
    for (int j = 0; j <= lmax; ++j)
      for (int k = cabs(i - j); k <= (i + j < lmax ? i + j : lmax); ++k) {
        if ((i + j + k) % 2) continue;
        if (i > LI || j > LE || k > LO) continue;
        t.l1[t.np] = i;
        t.l2[t.np] = j;
        t.l3[t.np] = k;
        t.np += 1;
      }
  int counts[16] = {};
  int offset_in_l[kMaxPaths] = {};
  for (int p = 0; p < t.np; ++p) {
    offset_in_l[p] = counts[t.l3[p]];
    counts[t.l3[p]] += 1;
  }
  int row_start[16] = {};
  int rows = 0;
  for (int l = 0; l <= lmax; ++l) {
    row_start[l] = rows;
    rows += counts[l] * (2 * l + 1);
  }
  t.out_rows = rows;
  int bond = 0, coef = 0;
  for (int p = 0; p < t.np; ++p) {
    int m1 = 2 * t.l1[p] + 1, m2 = 2 * t.l2[p] + 1, m3 = 2 * t.l3[p] + 1;
    t.bond_off[p] = bond;
    t.coef_off[p] = coef;
    t.out_row[p] = row_start[t.l3[p]] + offset_in_l[p] * m3;
    bond += m1 * m3;
    coef += m1 * m2 * m3;
  }
  t.bond_width = bond;
  t.coef_total = coef;
  return t;
}

template <int LI, int LE, int LO>
struct Paths {
  static constexpr PathTable T = make_paths(LI, LE, LO);
  static constexpr int NP = T.np;
  static constexpr int A = (LI + 1) * (LI + 1);  // input angular rows
  static constexpr int B = (LE + 1) * (LE + 1);  // harmonic width
  static constexpr int BW = T.bond_width;
  static constexpr int CT = T.coef_total;
  static constexpr int ROWS = T.out_rows;
};

// Compile-time loop: f(std::integral_constant<int, 0>) ... f(<N-1>).
template <class F, int... Is>
__device__ __forceinline__ void static_for_impl(F&& f, std::integer_sequence<int, Is...>) {
  (f(std::integral_constant<int, Is>{}), ...);
}
template <int N, class F>
__device__ __forceinline__ void static_for(F&& f) {
  static_for_impl(f, std::make_integer_sequence<int, N>{});
}

// Vector of CPL consecutive floats.
template <int CPL> struct Vec;
template <> struct Vec<1> { float v[1]; };
template <> struct Vec<2> { float v[2]; };
template <> struct Vec<4> { float v[4]; };

template <int CPL>
__device__ __forceinline__ void load_vec(float (&dst)[CPL], const float* __restrict__ src) {
  if constexpr (CPL == 4) {
    float4 t = __ldg(reinterpret_cast<const float4*>(src));
    dst[0] = t.x; dst[1] = t.y; dst[2] = t.z; dst[3] = t.w;
  } else if constexpr (CPL == 2) {
    float2 t = __ldg(reinterpret_cast<const float2*>(src));
    dst[0] = t.x; dst[1] = t.y;
  } else {
    dst[0] = __ldg(src);
  }
}

// Streaming (evict-first) load for data read exactly once.
template <int CPL>
__device__ __forceinline__ void load_vec_stream(float (&dst)[CPL], const float* __restrict__ src) {
  if constexpr (CPL == 4) {
    float4 t = __ldcs(reinterpret_cast<const float4*>(src));
    dst[0] = t.x; dst[1] = t.y; dst[2] = t.z; dst[3] = t.w;
  } else if constexpr (CPL == 2) {
    float2 t = __ldcs(reinterpret_cast<const float2*>(src));
    dst[0] = t.x; dst[1] = t.y;
  } else {
    dst[0] = __ldcs(src);
  }
}

template <int CPL>
__device__ __forceinline__ void store_vec_stream(float* __restrict__ dst, const float (&src)[CPL]) {
  if constexpr (CPL == 4) {
    __stcs(reinterpret_cast<float4*>(dst), make_float4(src[0], src[1], src[2], src[3]));
  } else if constexpr (CPL == 2) {
    __stcs(reinterpret_cast<float2*>(dst), make_float2(src[0], src[1]));
  } else {
    __stcs(dst, src[0]);
  }
}

template <int CPL>
__device__ __forceinline__ void store_vec(float* __restrict__ dst, const float (&src)[CPL]) {
  if constexpr (CPL == 4) {
    *reinterpret_cast<float4*>(dst) = make_float4(src[0], src[1], src[2], src[3]);
  } else if constexpr (CPL == 2) {
    *reinterpret_cast<float2*>(dst) = make_float2(src[0], src[1]);
  } else {
    dst[0] = src[0];
  }
}

// Bring one 128-byte line into L1 ahead of its use.
__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// Ask the bulk-copy unit to pull `bytes` at p into L2 (p 16-byte aligned, bytes a
// multiple of 16); one instruction per row, issued by the lane that owns the row.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Rows of `bytes` starting at base + r * bytes can be bulk-prefetched.
__device__ __forceinline__ bool bulk_rows(const void* base, uint32_t bytes) {
  return base != nullptr && ((reinterpret_cast<uintptr_t>(base) | bytes) & 15u) == 0;
}

}  // namespace ictc
