// Device building blocks shared by the standalone and graph-message TP kernels.
//
// Conventions
//   * A "unit" is one (node or instance, channel slice) pair handled by one warp;
//     lane t of slice s owns channels c0 .. c0+CPL-1 with c0 = (32 s + t) CPL.
//     Lanes with c0 >= C (channel tails) load and store nothing but still take
//     part in warp-wide work (bond construction, shuffles, barriers).
//   * The CG table is dense per bond column: value (p, i, k, j) sits at
//     coef_off[p] + (i m3 + k) m2 + j; bond column (p, i, k) = bond_off[p] + i m3 + k.
//   * Per warp shared memory: the instance's harmonics (32 floats) and its bond row.
#pragma once

#include "ictc_common.cuh"

namespace ictc {

struct TPArgs {
  const float* __restrict__ features;   // [rows_or_src_nodes, A*C]
  const float* __restrict__ harmonics;  // [E, B]
  const float* __restrict__ gates;      // [E, P*C] or null
  const float* __restrict__ weight;     // [P*C] or null
  const float* __restrict__ grad_out;   // [rows_or_dst_nodes, ROWS*C]
  const float* __restrict__ mask;       // [E] or null (graph only)
  const int64_t* __restrict__ src;      // [E] (graph only)
  const int64_t* __restrict__ dst;      // [E] (graph only)
  const int64_t* __restrict__ order;    // CSR edge order (graph only)
  const int64_t* __restrict__ offsets;  // CSR offsets [nodes+1] (graph only)
  float* __restrict__ out;
  float* __restrict__ grad_features;
  float* __restrict__ grad_harmonics;
  float* __restrict__ grad_gates;
  const float* __restrict__ coef;       // dense CG, [p][i][k][j]
  const int2* __restrict__ desc;        // per bond column: (yoff | m2 << 16, coef offset)
  int64_t rows;                         // instances (standalone) or CSR nodes (graph)
  int channels;
  int slices;                           // ceil(C / (32 * CPL))
  int stage_floats;                     // graph adjoint: per-warp staging buffer (0 = not staged)
  int* status;                          // device status word: non-zero after a timed-out wait
};

// Kernel parameters of the adjoint kernels: the launch arguments plus the dense
// CG table [p][i][k][j].  Passed by value (__grid_constant__), the coefficients
// sit in the constant parameter bank, so compile-time-indexed reads become
// FFMA constant operands instead of shared-memory loads.
template <int CT>
struct CoefParams {
  TPArgs a;
  float coef[CT];
};

constexpr int kWarps = 8;
// Graph kernels: how many edges ahead of the one being computed the gathered
// and streamed rows are pulled into L2.
constexpr int kAheadL2 = 4;
constexpr int kThreads = kWarps * 32;

__host__ __device__ constexpr int round4(int n) { return (n + 3) & ~3; }

template <class PS>
__host__ __device__ constexpr int table_floats() {
  return round4(PS::CT) + 2 * round4(PS::BW);  // coef + desc (int2 = 2 floats)
}
template <class PS>
__host__ __device__ constexpr int warp_floats() {
  return 32 + round4(PS::BW);  // harmonics row + bond row
}
template <class PS>
__host__ __device__ constexpr int smem_floats() {
  return table_floats<PS>() + kWarps * warp_floats<PS>() + kWarps * PS::B;  // + dY partials
}

// Graph adjoint staging area, after the kernel's regular shared memory: one
// mbarrier per warp (128 B), then one buffer of stage_floats per warp.
__host__ __device__ constexpr int stage_offset_bytes(int regular_bytes) { return (regular_bytes + 127) & ~127; }
__host__ __device__ constexpr int staged_smem_bytes(int regular_bytes, int stage_floats) {
  return stage_offset_bytes(regular_bytes) + 128 + kWarps * stage_floats * 4;
}
// Largest staged edge (output-gradient row + gate row) per warp.
constexpr int kStageBudgetBytes = 12288;
// Time limit of a staging wait.
constexpr uint64_t kStageWaitNs = 2000000000ull;

template <class PS>
__device__ __forceinline__ void load_tables(const TPArgs& a, float* s_coef, int2* s_desc) {
  for (int t = threadIdx.x; t < PS::CT; t += blockDim.x) s_coef[t] = a.coef[t];
  for (int t = threadIdx.x; t < PS::BW; t += blockDim.x) s_desc[t] = a.desc[t];
}

// bond[col] = sum_j C[col, j] * Y[yoff + j]   (cooperative over the warp)
template <class PS>
__device__ __forceinline__ void build_bond(const float* s_coef, const int2* s_desc, const float* s_y,
                                           float* s_bond, int lane) {
  for (int col = lane; col < PS::BW; col += 32) {
    const int2 d = s_desc[col];
    const int yoff = d.x & 0xffff;
    const int m2 = d.x >> 16;
    const float* cf = s_coef + d.y;
    float v = 0.f;
    for (int j = 0; j < m2; ++j) v = fmaf(cf[j], s_y[yoff + j], v);
    s_bond[col] = v;
  }
}

// Rows of one input degree l: x[i][ch] = feature (l, i, c0 + ch) of a packed row.
template <int l, int CPL, int LAYOUT>
__device__ __forceinline__ void load_degree(float (&x)[2 * l + 1][CPL], const float* row, int channels, int c0,
                                            bool active, bool stream) {
  constexpr int m = 2 * l + 1;
  if (!active) {
#pragma unroll
    for (int i = 0; i < m; ++i)
#pragma unroll
      for (int ch = 0; ch < CPL; ++ch) x[i][ch] = 0.f;
    return;
  }
  if constexpr (LAYOUT == kIrMul) {
#pragma unroll
    for (int i = 0; i < m; ++i) {
      const float* src = row + (int64_t)(l * l + i) * channels + c0;
      if (stream) load_vec_stream<CPL>(x[i], src);
      else load_vec<CPL>(x[i], src);
    }
  } else {
    const float* blk = row + l * l * channels;
#pragma unroll
    for (int ch = 0; ch < CPL; ++ch)
#pragma unroll
      for (int i = 0; i < m; ++i) x[i][ch] = __ldg(blk + (c0 + ch) * m + i);
  }
}

template <int l, int CPL, int LAYOUT>
__device__ __forceinline__ void store_degree(float* row, const float (&x)[2 * l + 1][CPL], int channels, int c0) {
  constexpr int m = 2 * l + 1;
  if constexpr (LAYOUT == kIrMul) {
#pragma unroll
    for (int i = 0; i < m; ++i) store_vec<CPL>(row + (int64_t)(l * l + i) * channels + c0, x[i]);
  } else {
#pragma unroll
    for (int ch = 0; ch < CPL; ++ch)
#pragma unroll
      for (int i = 0; i < m; ++i) row[l * l * channels + (c0 + ch) * m + i] = x[i][ch];
  }
}

template <int LI, int CPL, int LAYOUT>
__device__ __forceinline__ void load_features(float (&x)[(LI + 1) * (LI + 1)][CPL], const float* row,
                                              int channels, int c0, bool active, bool stream) {
  if (!active) {
#pragma unroll
    for (int r = 0; r < (LI + 1) * (LI + 1); ++r)
#pragma unroll
      for (int ch = 0; ch < CPL; ++ch) x[r][ch] = 0.f;
    return;
  }
  if constexpr (LAYOUT == kIrMul) {
#pragma unroll
    for (int r = 0; r < (LI + 1) * (LI + 1); ++r) {
      if (stream) load_vec_stream<CPL>(x[r], row + (int64_t)r * channels + c0);
      else load_vec<CPL>(x[r], row + (int64_t)r * channels + c0);
    }
  } else {
#pragma unroll
    for (int l = 0; l <= LI; ++l)
#pragma unroll
      for (int ch = 0; ch < CPL; ++ch)
#pragma unroll
        for (int i = 0; i < 2 * l + 1; ++i) x[l * l + i][ch] = __ldg(row + l * l * channels + (c0 + ch) * (2 * l + 1) + i);
  }
}

template <int LI, int CPL, int LAYOUT>
__device__ __forceinline__ void store_features(float* row, const float (&x)[(LI + 1) * (LI + 1)][CPL], int channels,
                                               int c0) {
  if constexpr (LAYOUT == kIrMul) {
#pragma unroll
    for (int r = 0; r < (LI + 1) * (LI + 1); ++r) store_vec<CPL>(row + (int64_t)r * channels + c0, x[r]);
  } else {
#pragma unroll
    for (int l = 0; l <= LI; ++l)
#pragma unroll
      for (int ch = 0; ch < CPL; ++ch)
#pragma unroll
        for (int i = 0; i < 2 * l + 1; ++i) row[l * l * channels + (c0 + ch) * (2 * l + 1) + i] = x[l * l + i][ch];
  }
}

// Vector load of CPL consecutive floats from shared memory.
template <int CPL>
__device__ __forceinline__ void load_vec_shared(float (&dst)[CPL], const float* src) {
  if constexpr (CPL == 4) {
    const float4 t = *reinterpret_cast<const float4*>(src);
    dst[0] = t.x; dst[1] = t.y; dst[2] = t.z; dst[3] = t.w;
  } else if constexpr (CPL == 2) {
    const float2 t = *reinterpret_cast<const float2*>(src);
    dst[0] = t.x; dst[1] = t.y;
  } else {
    dst[0] = src[0];
  }
}

// The m3 x CPL output block of one path from a packed output row staged in
// shared memory.  mul_ir: the lane's CPL channels are 2 m3 consecutive floats,
// read as float2 (c0 and the block offset are even when CPL = 2).
template <int CPL, int LAYOUT, int RO, int m3>
__device__ __forceinline__ void load_out_block_shared(float (&G)[m3][CPL], const float* row, int channels,
                                                      int c0) {
  if constexpr (LAYOUT == kIrMul) {
#pragma unroll
    for (int k = 0; k < m3; ++k) load_vec_shared<CPL>(G[k], row + (RO + k) * channels + c0);
  } else if constexpr (CPL == 2) {
    const float* blk = row + RO * channels + c0 * m3;
    float t[2 * m3];
#pragma unroll
    for (int q = 0; q < m3; ++q) {
      const float2 v = *reinterpret_cast<const float2*>(blk + 2 * q);
      t[2 * q] = v.x;
      t[2 * q + 1] = v.y;
    }
#pragma unroll
    for (int ch = 0; ch < 2; ++ch)
#pragma unroll
      for (int k = 0; k < m3; ++k) G[k][ch] = t[ch * m3 + k];
  } else {
#pragma unroll
    for (int ch = 0; ch < CPL; ++ch)
#pragma unroll
      for (int k = 0; k < m3; ++k) G[k][ch] = row[RO * channels + (c0 + ch) * m3 + k];
  }
}

// All input rows of the lane's channels from a packed feature row staged in
// shared memory (mul_ir, CPL = 2: float2 reads of each degree's 2 m floats).
template <int LI, int CPL, int LAYOUT>
__device__ __forceinline__ void load_features_shared(float (&x)[(LI + 1) * (LI + 1)][CPL], const float* row,
                                                     int channels, int c0, bool active) {
  if (!active) {
#pragma unroll
    for (int r = 0; r < (LI + 1) * (LI + 1); ++r)
#pragma unroll
      for (int ch = 0; ch < CPL; ++ch) x[r][ch] = 0.f;
    return;
  }
  if constexpr (LAYOUT == kIrMul) {
#pragma unroll
    for (int r = 0; r < (LI + 1) * (LI + 1); ++r) load_vec_shared<CPL>(x[r], row + r * channels + c0);
  } else {
    static_for<LI + 1>([&](auto lc) {
      constexpr int l = decltype(lc)::value, m = 2 * l + 1;
      const float* blk = row + l * l * channels + c0 * m;
      if constexpr (CPL == 2) {
        float t[2 * m];
#pragma unroll
        for (int q = 0; q < m; ++q) {
          const float2 v = *reinterpret_cast<const float2*>(blk + 2 * q);
          t[2 * q] = v.x;
          t[2 * q + 1] = v.y;
        }
#pragma unroll
        for (int ch = 0; ch < 2; ++ch)
#pragma unroll
          for (int i = 0; i < m; ++i) x[l * l + i][ch] = t[ch * m + i];
      } else {
#pragma unroll
        for (int ch = 0; ch < CPL; ++ch)
#pragma unroll
          for (int i = 0; i < m; ++i) x[l * l + i][ch] = blk[ch * m + i];
      }
    });
  }
}

// Load the m3 x CPL output block of one path from a packed output row.
template <int CPL, int LAYOUT, int RO, int m3>
__device__ __forceinline__ void load_out_block(float (&G)[m3][CPL], const float* row, int channels, int c0,
                                               bool stream) {
  if constexpr (LAYOUT == kIrMul) {
#pragma unroll
    for (int k = 0; k < m3; ++k) {
      if (stream) load_vec_stream<CPL>(G[k], row + (int64_t)(RO + k) * channels + c0);
      else load_vec<CPL>(G[k], row + (int64_t)(RO + k) * channels + c0);
    }
  } else {
#pragma unroll
    for (int ch = 0; ch < CPL; ++ch)
#pragma unroll
      for (int k = 0; k < m3; ++k) G[k][ch] = __ldg(row + (int64_t)RO * channels + (c0 + ch) * m3 + k);
  }
}

// Named barrier over the `count` threads of one warp group (id 1..15).
__device__ __forceinline__ void group_barrier(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Sum of v over the 32 lanes, returned on every lane.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace ictc
