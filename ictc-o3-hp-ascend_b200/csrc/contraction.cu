// MACE symmetric contraction on sm_100a, evaluated as a per-node polynomial.
//
// The reference recursion (ictc_o3/ops/_mace_symmetric_contraction.py:298-346,
// with U from ictc_o3/basis/ictd_irreps.py:1465-1517) computes, per node n of
// species s, channel c and target degree t,
//   out[m] = sum_nu sum_{i1..inu} U_nu[m, i1..inu, p] W_nu[s, p, c] x_{i1} .. x_{inu}.
// Symmetrising U over its input axes turns this into a polynomial over the
// monomials x_i, x_i x_j (i <= j), x_i x_j x_k (i <= j <= k).  The host folds
// the species weights into one coefficient table (a GEMM, T = Usym W):
//   T[s][t][row][m][c],  rows in the traversal order
//     for i: (i) ; for j >= i: (i,j) ; for k >= j: (i,j,k)
// restricted to the orders present (correlation 1..3).
//
// Work decomposition: a warp owns a tile of NB nodes of one species (the host
// builds species-homogeneous tiles) and a 32-channel slice; lane = channel.
// Every coefficient row is one coalesced 128-B load reused for the NB nodes.
// Node inputs are staged in shared memory ([node][d][lane], conflict-free);
// the feature gradient accumulates in shared memory columns owned by a single
// lane each, so no atomics are needed.
#include "ictc_common.cuh"
#include "ictc_cuda.h"

#include <cstdio>

void ictc_set_error(const char* fmt, const char* detail);

namespace ictc {

// Nodes per tile (NB): every coefficient row streamed from L2 serves NB nodes, so the
// table traffic per node falls as 1/NB (the kernels are bound by that stream).
constexpr int kScNodes = 8;
// Warps per CTA: the staged inputs (and gradients) take NB * D * 32 floats per warp;
// static shared memory stays under 48 KB.
__host__ __device__ constexpr int sc_warps(int D) { return D > 9 ? 1 : 2; }

struct SCArgs {
  const float* __restrict__ x;          // [N, C*D] mul_ir flat
  const float* __restrict__ table;      // [S, R, C]
  const int64_t* __restrict__ tiles;    // [num_tiles, NB], -1 padded
  const int32_t* __restrict__ tile_species;
  const float* __restrict__ grad_out;   // [N, C*sum_t M_t]
  float* __restrict__ out;              // [N, C*sum_t M_t]
  float* __restrict__ grad_x;           // [N, C*D]
  const float* __restrict__ dir;        // [N, C*D] direction h of the second-order kernels
  int64_t num_tiles;
  int channels;
  int targets;                          // target_lmax + 1
  int64_t rows;                         // R (per species)
};

__host__ __device__ constexpr int sc_monomials(int D, int corr) {
  int k = 0;
  if (corr >= 1) k += D;
  if (corr >= 2) k += D * (D + 1) / 2;
  if (corr >= 3) k += D * (D + 1) * (D + 2) / 6;
  return k;
}

template <int D>
__device__ __forceinline__ void stage_inputs(const SCArgs& a, float (*s_x)[D][32], const int64_t* nodes, int c,
                                             bool active) {
  // s_x[n][d][lane] = x[node][l^2 C + c (2l+1) + i], d = l^2 + i.
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int n = 0; n < kScNodes; ++n) {
    const int64_t node = nodes[n];
#pragma unroll
    for (int l = 0; l * l < D; ++l) {
      const int m = 2 * l + 1;
#pragma unroll
      for (int i = 0; i < m; ++i)
        s_x[n][l * l + i][lane] =
            (node >= 0 && active) ? __ldg(a.x + node * (int64_t)a.channels * D + l * l * a.channels + c * m + i) : 0.f;
    }
  }
}

// The same staging for another [N, C*D] array (the direction h).
template <int D>
__device__ __forceinline__ void stage_array(const float* src, int channels, float (*s_v)[D][32],
                                            const int64_t* nodes, int c, bool active) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int n = 0; n < kScNodes; ++n) {
    const int64_t node = nodes[n];
#pragma unroll
    for (int l = 0; l * l < D; ++l) {
      const int m = 2 * l + 1;
#pragma unroll
      for (int i = 0; i < m; ++i)
        s_v[n][l * l + i][lane] =
            (node >= 0 && active) ? __ldg(src + node * (int64_t)channels * D + l * l * channels + c * m + i) : 0.f;
    }
  }
}

template <int D, int CORR>
__global__ void __launch_bounds__(128) sc_forward_kernel(SCArgs a) {
  constexpr int kScWarps = sc_warps(D);
  __shared__ float s_x_all[kScWarps][kScNodes][D][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float (*s_x)[D][32] = s_x_all[warp];
  const int C = a.channels;
  const int slices = (C + 31) / 32;
  const int64_t units = a.num_tiles * slices;
  for (int64_t unit = (int64_t)blockIdx.x * kScWarps + warp; unit < units; unit += (int64_t)gridDim.x * kScWarps) {
    const int64_t tile = unit / slices;
    const int c = (int)(unit - tile * slices) * 32 + lane;
    const bool active = c < C;
    int64_t nodes[kScNodes];
#pragma unroll
    for (int n = 0; n < kScNodes; ++n) nodes[n] = a.tiles[tile * kScNodes + n];
    __syncwarp();
    stage_inputs<D>(a, s_x, nodes, c, active);
    __syncwarp();
    const float* tab = a.table + (int64_t)a.tile_species[tile] * a.rows * C + (active ? c : 0);
    int64_t out_col = 0;  // first output column of the target block (channels * sum M)
    for (int t = 0; t < a.targets; ++t) {
      const int M = 2 * t + 1;
      float acc[kScNodes][7];
#pragma unroll
      for (int n = 0; n < kScNodes; ++n)
#pragma unroll
        for (int m = 0; m < 7; ++m) acc[n][m] = 0.f;
      auto row = [&](const float (&mono)[kScNodes]) {
#pragma unroll
        for (int m = 0; m < 7; ++m) {
          if (m < M) {
            const float coef = __ldg(tab);
            tab += C;
#pragma unroll
            for (int n = 0; n < kScNodes; ++n) acc[n][m] = fmaf(coef, mono[n], acc[n][m]);
          }
        }
      };
#pragma unroll 1
      for (int i = 0; i < D; ++i) {
        float xi[kScNodes];
#pragma unroll
        for (int n = 0; n < kScNodes; ++n) xi[n] = s_x[n][i][lane];
        if (CORR >= 1) row(xi);
        if (CORR >= 2) {
#pragma unroll 1
          for (int j = i; j < D; ++j) {
            float xij[kScNodes];
#pragma unroll
            for (int n = 0; n < kScNodes; ++n) xij[n] = xi[n] * s_x[n][j][lane];
            row(xij);
            if (CORR >= 3) {
#pragma unroll 1
              for (int k = j; k < D; ++k) {
                float xijk[kScNodes];
#pragma unroll
                for (int n = 0; n < kScNodes; ++n) xijk[n] = xij[n] * s_x[n][k][lane];
                row(xijk);
              }
            }
          }
        }
      }
      if (active) {
#pragma unroll
        for (int n = 0; n < kScNodes; ++n) {
          if (nodes[n] < 0) continue;
          float* dst = a.out + nodes[n] * (int64_t)C * (a.targets * a.targets) + out_col + c * M;
#pragma unroll
          for (int m = 0; m < 7; ++m)
            if (m < M) dst[m] = acc[n][m];
        }
      }
      out_col += (int64_t)C * M;
    }
  }
}

// Feature gradient: dx_i = sum_t sum_m G_t[m] d out_t[m] / d x_i.
template <int D, int CORR>
__global__ void __launch_bounds__(128) sc_backward_kernel(SCArgs a) {
  constexpr int kScWarps = sc_warps(D);
  __shared__ float s_x_all[kScWarps][kScNodes][D][32];
  __shared__ float s_dx_all[kScWarps][kScNodes][D][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float (*s_x)[D][32] = s_x_all[warp];
  float (*s_dx)[D][32] = s_dx_all[warp];
  const int C = a.channels;
  const int slices = (C + 31) / 32;
  const int64_t units = a.num_tiles * slices;
  const int64_t out_width = (int64_t)C * a.targets * a.targets;
  for (int64_t unit = (int64_t)blockIdx.x * kScWarps + warp; unit < units; unit += (int64_t)gridDim.x * kScWarps) {
    const int64_t tile = unit / slices;
    const int c = (int)(unit - tile * slices) * 32 + lane;
    const bool active = c < C;
    int64_t nodes[kScNodes];
#pragma unroll
    for (int n = 0; n < kScNodes; ++n) nodes[n] = a.tiles[tile * kScNodes + n];
    __syncwarp();
    stage_inputs<D>(a, s_x, nodes, c, active);
#pragma unroll
    for (int n = 0; n < kScNodes; ++n)
#pragma unroll
      for (int d = 0; d < D; ++d) s_dx[n][d][lane] = 0.f;
    __syncwarp();
    const float* tab = a.table + (int64_t)a.tile_species[tile] * a.rows * C + (active ? c : 0);
    int64_t out_col = 0;
    for (int t = 0; t < a.targets; ++t) {
      const int M = 2 * t + 1;
      float g[kScNodes][7];
#pragma unroll
      for (int n = 0; n < kScNodes; ++n)
#pragma unroll
        for (int m = 0; m < 7; ++m)
          g[n][m] = (m < M && nodes[n] >= 0 && active) ? __ldg(a.grad_out + nodes[n] * out_width + out_col + c * M + m)
                                                       : 0.f;
      // a[n] = sum_m T[row][m] g[n][m] for the current row
      auto project = [&](float (&av)[kScNodes]) {
#pragma unroll
        for (int n = 0; n < kScNodes; ++n) av[n] = 0.f;
#pragma unroll
        for (int m = 0; m < 7; ++m) {
          if (m < M) {
            const float coef = __ldg(tab);
            tab += C;
#pragma unroll
            for (int n = 0; n < kScNodes; ++n) av[n] = fmaf(coef, g[n][m], av[n]);
          }
        }
      };
#pragma unroll 1
      for (int i = 0; i < D; ++i) {
        float xi[kScNodes], dxi[kScNodes];
#pragma unroll
        for (int n = 0; n < kScNodes; ++n) { xi[n] = s_x[n][i][lane]; dxi[n] = 0.f; }
        if (CORR >= 1) {
          float av[kScNodes];
          project(av);
#pragma unroll
          for (int n = 0; n < kScNodes; ++n) dxi[n] += av[n];
        }
        if (CORR >= 2) {
#pragma unroll 1
          for (int j = i; j < D; ++j) {
            float xj[kScNodes], dxj[kScNodes];
#pragma unroll
            for (int n = 0; n < kScNodes; ++n) { xj[n] = s_x[n][j][lane]; dxj[n] = 0.f; }
            {
              // d(x_i x_j): x_j towards i, x_i towards j (both when i == j: 2 x_i).
              float av[kScNodes];
              project(av);
#pragma unroll
              for (int n = 0; n < kScNodes; ++n) {
                dxi[n] = fmaf(av[n], xj[n], dxi[n]);
                dxj[n] = fmaf(av[n], xi[n], dxj[n]);
              }
            }
            if (CORR >= 3) {
              // Unrolled: the table loads of several monomials are in flight at once
              // (the loop is L2-latency-bound; 19.1 -> 15.3 ms per MD step at D = 9).
#pragma unroll 4
              for (int k = j; k < D; ++k) {
                float av[kScNodes];
                project(av);
#pragma unroll
                for (int n = 0; n < kScNodes; ++n) {
                  const float xk = s_x[n][k][lane];
                  dxi[n] = fmaf(av[n], xj[n] * xk, dxi[n]);
                  dxj[n] = fmaf(av[n], xi[n] * xk, dxj[n]);
                  s_dx[n][k][lane] = fmaf(av[n], xi[n] * xj[n], s_dx[n][k][lane]);
                }
              }
            }
#pragma unroll
            for (int n = 0; n < kScNodes; ++n) s_dx[n][j][lane] += dxj[n];
          }
        }
#pragma unroll
        for (int n = 0; n < kScNodes; ++n) s_dx[n][i][lane] += dxi[n];
      }
      out_col += (int64_t)C * M;
    }
    if (active) {
#pragma unroll
      for (int n = 0; n < kScNodes; ++n) {
        if (nodes[n] < 0) continue;
        float* dst = a.grad_x + nodes[n] * (int64_t)C * D;
#pragma unroll
        for (int l = 0; l * l < D; ++l) {
          const int m = 2 * l + 1;
#pragma unroll
          for (int i = 0; i < m; ++i) dst[l * l * C + c * m + i] = s_dx[n][l * l + i][lane];
        }
      }
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Second order (force-loss training).  With the directional monomials
//   (h.grad) x_i = h_i,  (h.grad) x_i x_j = h_i x_j + x_i h_j,
//   (h.grad) x_i x_j x_k = h_i x_j x_k + x_i h_j x_k + x_i x_j h_k,
// sc_directional_kernel evaluates F[m] = sum_r T[r][m] (h.grad) mono_r(x) (the
// derivative of the feature gradient with respect to the output cotangent), and
// sc_hvp_kernel the gradient of sum_m g_m F[m] with respect to x (a Hessian-vector
// product of the polynomial).  Same tiles, lanes and table stream as the first-
// order kernels.
// ---------------------------------------------------------------------------
template <int D, int CORR>
__global__ void __launch_bounds__(128) sc_directional_kernel(SCArgs a) {
  constexpr int kScWarps = sc_warps(D);
  __shared__ float s_x_all[kScWarps][kScNodes][D][32];
  __shared__ float s_h_all[kScWarps][kScNodes][D][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float (*s_x)[D][32] = s_x_all[warp];
  float (*s_h)[D][32] = s_h_all[warp];
  const int C = a.channels;
  const int slices = (C + 31) / 32;
  const int64_t units = a.num_tiles * slices;
  for (int64_t unit = (int64_t)blockIdx.x * kScWarps + warp; unit < units; unit += (int64_t)gridDim.x * kScWarps) {
    const int64_t tile = unit / slices;
    const int c = (int)(unit - tile * slices) * 32 + lane;
    const bool active = c < C;
    int64_t nodes[kScNodes];
#pragma unroll
    for (int n = 0; n < kScNodes; ++n) nodes[n] = a.tiles[tile * kScNodes + n];
    __syncwarp();
    stage_inputs<D>(a, s_x, nodes, c, active);
    stage_array<D>(a.dir, C, s_h, nodes, c, active);
    __syncwarp();
    const float* tab = a.table + (int64_t)a.tile_species[tile] * a.rows * C + (active ? c : 0);
    int64_t out_col = 0;
    for (int t = 0; t < a.targets; ++t) {
      const int M = 2 * t + 1;
      float acc[kScNodes][7];
#pragma unroll
      for (int n = 0; n < kScNodes; ++n)
#pragma unroll
        for (int m = 0; m < 7; ++m) acc[n][m] = 0.f;
      auto row = [&](const float (&v)[kScNodes]) {
#pragma unroll
        for (int m = 0; m < 7; ++m) {
          if (m < M) {
            const float coef = __ldg(tab);
            tab += C;
#pragma unroll
            for (int n = 0; n < kScNodes; ++n) acc[n][m] = fmaf(coef, v[n], acc[n][m]);
          }
        }
      };
#pragma unroll 1
      for (int i = 0; i < D; ++i) {
        float xi[kScNodes], hi[kScNodes];
#pragma unroll
        for (int n = 0; n < kScNodes; ++n) { xi[n] = s_x[n][i][lane]; hi[n] = s_h[n][i][lane]; }
        if (CORR >= 1) row(hi);
        if (CORR >= 2) {
#pragma unroll 1
          for (int j = i; j < D; ++j) {
            float xij[kScNodes], dij[kScNodes];
#pragma unroll
            for (int n = 0; n < kScNodes; ++n) {
              const float xj = s_x[n][j][lane], hj = s_h[n][j][lane];
              xij[n] = xi[n] * xj;
              dij[n] = fmaf(hi[n], xj, xi[n] * hj);
            }
            row(dij);
            if (CORR >= 3) {
#pragma unroll 4
              for (int k = j; k < D; ++k) {
                float dijk[kScNodes];
#pragma unroll
                for (int n = 0; n < kScNodes; ++n) dijk[n] = fmaf(dij[n], s_x[n][k][lane], xij[n] * s_h[n][k][lane]);
                row(dijk);
              }
            }
          }
        }
      }
      if (active) {
#pragma unroll
        for (int n = 0; n < kScNodes; ++n) {
          if (nodes[n] < 0) continue;
          float* dst = a.out + nodes[n] * (int64_t)C * (a.targets * a.targets) + out_col + c * M;
#pragma unroll
          for (int m = 0; m < 7; ++m)
            if (m < M) dst[m] = acc[n][m];
        }
      }
      out_col += (int64_t)C * M;
    }
  }
}

// Gradient with respect to x of sum_t sum_m g_t[m] F_t[m] (F as in
// sc_directional_kernel): for each monomial row, av = sum_m T[row][m] g[m] and
//   (i,j):   d/dx_i += av h_j,              d/dx_j += av h_i
//   (i,j,k): d/dx_i += av (h_j x_k + x_j h_k), d/dx_j += av (h_i x_k + x_i h_k),
//            d/dx_k += av (h_i x_j + x_i h_j)
// (first-order rows are linear in x: no contribution).  One warp per CTA keeps the
// three staged arrays inside the static shared-memory limit.
template <int D, int CORR>
__global__ void __launch_bounds__(64) sc_hvp_kernel(SCArgs a) {
  constexpr int kW = D > 4 ? 1 : 2;
  __shared__ float s_x_all[kW][kScNodes][D][32];
  __shared__ float s_h_all[kW][kScNodes][D][32];
  __shared__ float s_dx_all[kW][kScNodes][D][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float (*s_x)[D][32] = s_x_all[warp];
  float (*s_h)[D][32] = s_h_all[warp];
  float (*s_dx)[D][32] = s_dx_all[warp];
  const int C = a.channels;
  const int slices = (C + 31) / 32;
  const int64_t units = a.num_tiles * slices;
  const int64_t out_width = (int64_t)C * a.targets * a.targets;
  for (int64_t unit = (int64_t)blockIdx.x * kW + warp; unit < units; unit += (int64_t)gridDim.x * kW) {
    const int64_t tile = unit / slices;
    const int c = (int)(unit - tile * slices) * 32 + lane;
    const bool active = c < C;
    int64_t nodes[kScNodes];
#pragma unroll
    for (int n = 0; n < kScNodes; ++n) nodes[n] = a.tiles[tile * kScNodes + n];
    __syncwarp();
    stage_inputs<D>(a, s_x, nodes, c, active);
    stage_array<D>(a.dir, C, s_h, nodes, c, active);
#pragma unroll
    for (int n = 0; n < kScNodes; ++n)
#pragma unroll
      for (int d = 0; d < D; ++d) s_dx[n][d][lane] = 0.f;
    __syncwarp();
    const float* tab = a.table + (int64_t)a.tile_species[tile] * a.rows * C + (active ? c : 0);
    int64_t out_col = 0;
    for (int t = 0; t < a.targets; ++t) {
      const int M = 2 * t + 1;
      float g[kScNodes][7];
#pragma unroll
      for (int n = 0; n < kScNodes; ++n)
#pragma unroll
        for (int m = 0; m < 7; ++m)
          g[n][m] = (m < M && nodes[n] >= 0 && active) ? __ldg(a.grad_out + nodes[n] * out_width + out_col + c * M + m)
                                                       : 0.f;
      auto project = [&](float (&av)[kScNodes]) {
#pragma unroll
        for (int n = 0; n < kScNodes; ++n) av[n] = 0.f;
#pragma unroll
        for (int m = 0; m < 7; ++m) {
          if (m < M) {
            const float coef = __ldg(tab);
            tab += C;
#pragma unroll
            for (int n = 0; n < kScNodes; ++n) av[n] = fmaf(coef, g[n][m], av[n]);
          }
        }
      };
#pragma unroll 1
      for (int i = 0; i < D; ++i) {
        float xi[kScNodes], hi[kScNodes], dxi[kScNodes];
#pragma unroll
        for (int n = 0; n < kScNodes; ++n) { xi[n] = s_x[n][i][lane]; hi[n] = s_h[n][i][lane]; dxi[n] = 0.f; }
        if (CORR >= 1) tab += (int64_t)M * C;          // linear rows: no second derivative
        if (CORR >= 2) {
#pragma unroll 1
          for (int j = i; j < D; ++j) {
            float xj[kScNodes], hj[kScNodes], dxj[kScNodes];
#pragma unroll
            for (int n = 0; n < kScNodes; ++n) { xj[n] = s_x[n][j][lane]; hj[n] = s_h[n][j][lane]; dxj[n] = 0.f; }
            {
              float av[kScNodes];
              project(av);
#pragma unroll
              for (int n = 0; n < kScNodes; ++n) {
                dxi[n] = fmaf(av[n], hj[n], dxi[n]);
                dxj[n] = fmaf(av[n], hi[n], dxj[n]);
              }
            }
            if (CORR >= 3) {
#pragma unroll 4
              for (int k = j; k < D; ++k) {
                float av[kScNodes];
                project(av);
#pragma unroll
                for (int n = 0; n < kScNodes; ++n) {
                  const float xk = s_x[n][k][lane], hk = s_h[n][k][lane];
                  dxi[n] = fmaf(av[n], fmaf(hj[n], xk, xj[n] * hk), dxi[n]);
                  dxj[n] = fmaf(av[n], fmaf(hi[n], xk, xi[n] * hk), dxj[n]);
                  s_dx[n][k][lane] = fmaf(av[n], fmaf(hi[n], xj[n], xi[n] * hj[n]), s_dx[n][k][lane]);
                }
              }
            }
#pragma unroll
            for (int n = 0; n < kScNodes; ++n) s_dx[n][j][lane] += dxj[n];
          }
        }
#pragma unroll
        for (int n = 0; n < kScNodes; ++n) s_dx[n][i][lane] += dxi[n];
      }
      out_col += (int64_t)C * M;
    }
    if (active) {
#pragma unroll
      for (int n = 0; n < kScNodes; ++n) {
        if (nodes[n] < 0) continue;
        float* dst = a.grad_x + nodes[n] * (int64_t)C * D;
#pragma unroll
        for (int l = 0; l * l < D; ++l) {
          const int m = 2 * l + 1;
#pragma unroll
          for (int i = 0; i < m; ++i) dst[l * l * C + c * m + i] = s_dx[n][l * l + i][lane];
        }
      }
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Table gradient of one target t:
//   dT[s][row0 + r*M + m][c] = sum_{nodes n of species s} g_t[n][c][m] v_r(n, c)
// with v_r = mono_r(x) or, given a direction h, (h.grad) mono_r(x).  A warp owns
// (species, 32 channels, a block of RB = 64 / M monomial rows) and walks every
// tile of its species (tiles are grouped by species), accumulating in registers:
// deterministic, no atomics.  The (i, j, k) of every row sit in shared memory.
// ---------------------------------------------------------------------------
struct SCGradArgs {
  const float* __restrict__ x;          // [N, C*D]
  const float* __restrict__ dir;        // [N, C*D] or null
  const float* __restrict__ grad_out;   // [N, C*sum_t M_t]
  const int64_t* __restrict__ tiles;
  const int32_t* __restrict__ tile_species;
  float* __restrict__ grad_table;       // [S, R_total, C]
  int64_t num_tiles, rows_total, row0;  // table rows per species, first row of target t
  int channels, targets, target, species, monomials;
  int64_t out_col;                      // C * sum_{t' < t} M_t'
};

template <int D, int CORR, int M>
__global__ void __launch_bounds__(128) sc_table_grad_kernel(SCGradArgs a) {
  constexpr int RB = 64 / M;
  // (i, j, k) of every monomial row; an absent factor points at slot D, which holds
  // x = 1 and h = 0 in the staged node row.
  __shared__ int s_mono[sc_monomials(16, 3)];
  __shared__ float s_x[4][D + 1][32];
  __shared__ float s_h[4][D + 1][32];
  if (threadIdx.x == 0) {
    int r = 0;
    for (int i = 0; i < D; ++i) {
      if (CORR >= 1) s_mono[r++] = i | (D << 8) | (D << 16);
      if (CORR >= 2)
        for (int j = i; j < D; ++j) {
          s_mono[r++] = i | (j << 8) | (D << 16);
          if (CORR >= 3)
            for (int k = j; k < D; ++k) s_mono[r++] = i | (j << 8) | (k << 16);
        }
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = a.channels;
  const int slices = (C + 31) / 32;
  const int blocks_r = (a.monomials + RB - 1) / RB;
  const int64_t unit = (int64_t)blockIdx.x * 4 + warp;
  if (unit >= (int64_t)a.species * slices * blocks_r) return;
  const int s = (int)(unit / ((int64_t)slices * blocks_r));
  const int rem = (int)(unit - (int64_t)s * slices * blocks_r);
  const int cs = rem / blocks_r, rb = rem - cs * blocks_r;
  const int c = cs * 32 + lane;
  const bool active = c < C;
  const int r0 = rb * RB;
  // tiles of species s: [lo, hi) in the species-sorted tile list (binary searches)
  int64_t lo = 0, hi = a.num_tiles;
  {
    int64_t l = 0, h = a.num_tiles;
    while (l < h) { const int64_t mid = (l + h) / 2; if (a.tile_species[mid] < s) l = mid + 1; else h = mid; }
    lo = l;
    h = a.num_tiles;
    while (l < h) { const int64_t mid = (l + h) / 2; if (a.tile_species[mid] <= s) l = mid + 1; else h = mid; }
    hi = l;
  }
  float (*xs)[32] = s_x[warp];
  float (*hs)[32] = s_h[warp];
  xs[D][lane] = 1.f;
  hs[D][lane] = 0.f;
  float acc[RB][M];
#pragma unroll
  for (int q = 0; q < RB; ++q)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[q][m] = 0.f;
  const int64_t out_width = (int64_t)C * a.targets * a.targets;
  for (int64_t tile = lo; tile < hi; ++tile) {
#pragma unroll 1
    for (int n = 0; n < kScNodes; ++n) {
      const int64_t node = a.tiles[tile * kScNodes + n];   // warp-uniform
      if (node < 0) continue;
      const float* xr = a.x + node * (int64_t)C * D;
      const float* hr = a.dir ? a.dir + node * (int64_t)C * D : nullptr;
      __syncwarp();
#pragma unroll
      for (int l = 0; l * l < D; ++l)
#pragma unroll
        for (int i = 0; i < 2 * l + 1; ++i) {
          xs[l * l + i][lane] = active ? __ldg(xr + l * l * C + c * (2 * l + 1) + i) : 0.f;
          hs[l * l + i][lane] = (active && hr) ? __ldg(hr + l * l * C + c * (2 * l + 1) + i) : 0.f;
        }
      float g[M];
#pragma unroll
      for (int m = 0; m < M; ++m) g[m] = active ? __ldg(a.grad_out + node * out_width + a.out_col + c * M + m) : 0.f;
      __syncwarp();
#pragma unroll
      for (int q = 0; q < RB; ++q) {
        const int r = r0 + q;
        if (r < a.monomials) {
          const int code = s_mono[r];
          const int i = code & 255, j = (code >> 8) & 255, k = (code >> 16) & 255;
          const float xi = xs[i][lane], xj = xs[j][lane], xk = xs[k][lane];
          // (h.grad)(x_i x_j x_k); absent factors have x = 1, h = 0
          const float v = a.dir ? fmaf(hs[i][lane], xj * xk, xi * fmaf(hs[j][lane], xk, xj * hs[k][lane]))
                                : xi * xj * xk;
#pragma unroll
          for (int m = 0; m < M; ++m) acc[q][m] = fmaf(g[m], v, acc[q][m]);
        }
      }
    }
  }
  if (!active) return;
  float* dst = a.grad_table + ((int64_t)s * a.rows_total + a.row0) * C + c;
#pragma unroll
  for (int q = 0; q < RB; ++q) {
    const int r = r0 + q;
    if (r < a.monomials) {
#pragma unroll
      for (int m = 0; m < M; ++m) dst[((int64_t)r * M + m) * C] = acc[q][m];
    }
  }
}

using SCFn = void (*)(SCArgs);

static SCFn sc_kernel(int lmax, int corr, bool backward) {
#define ICTC_SC_CASE(L, CO)                                                                      \
  if (lmax == L && corr == CO)                                                                   \
    return backward ? sc_backward_kernel<(L + 1) * (L + 1), CO> : sc_forward_kernel<(L + 1) * (L + 1), CO>;
  ICTC_SC_CASE(1, 1) ICTC_SC_CASE(1, 2) ICTC_SC_CASE(1, 3)
  ICTC_SC_CASE(2, 1) ICTC_SC_CASE(2, 2) ICTC_SC_CASE(2, 3)
  ICTC_SC_CASE(3, 1) ICTC_SC_CASE(3, 2) ICTC_SC_CASE(3, 3)
#undef ICTC_SC_CASE
  return nullptr;
}

// Second-order kernels: kind 0 = directional polynomial, 1 = Hessian-vector product.
static SCFn sc_kernel2(int lmax, int corr, int kind, int* warps) {
  const int D = (lmax + 1) * (lmax + 1);
  *warps = kind == 0 ? sc_warps(D) : (D > 4 ? 1 : 2);
#define ICTC_SC2_CASE(L, CO)                                                                    \
  if (lmax == L && corr == CO)                                                                  \
    return kind == 0 ? sc_directional_kernel<(L + 1) * (L + 1), CO> : sc_hvp_kernel<(L + 1) * (L + 1), CO>;
  ICTC_SC2_CASE(1, 1) ICTC_SC2_CASE(1, 2) ICTC_SC2_CASE(1, 3)
  ICTC_SC2_CASE(2, 1) ICTC_SC2_CASE(2, 2) ICTC_SC2_CASE(2, 3)
  ICTC_SC2_CASE(3, 1) ICTC_SC2_CASE(3, 2) ICTC_SC2_CASE(3, 3)
#undef ICTC_SC2_CASE
  return nullptr;
}

using SCGradFn = void (*)(SCGradArgs);

template <int D, int CO>
static SCGradFn sc_grad_for_m(int M) {
  switch (M) {
    case 1: return sc_table_grad_kernel<D, CO, 1>;
    case 3: return sc_table_grad_kernel<D, CO, 3>;
    case 5: return sc_table_grad_kernel<D, CO, 5>;
    case 7: return sc_table_grad_kernel<D, CO, 7>;
    default: return nullptr;
  }
}

static SCGradFn sc_grad_kernel(int lmax, int corr, int M) {
#define ICTC_SCG_CASE(L, CO) \
  if (lmax == L && corr == CO) return sc_grad_for_m<(L + 1) * (L + 1), CO>(M);
  ICTC_SCG_CASE(1, 1) ICTC_SCG_CASE(1, 2) ICTC_SCG_CASE(1, 3)
  ICTC_SCG_CASE(2, 1) ICTC_SCG_CASE(2, 2) ICTC_SCG_CASE(2, 3)
  ICTC_SCG_CASE(3, 1) ICTC_SCG_CASE(3, 2) ICTC_SCG_CASE(3, 3)
#undef ICTC_SCG_CASE
  return nullptr;
}

// ---------------------------------------------------------------------------
// Weight fold of one target degree: T[s, row0 + r, c] = sum_p U[r, p] W[s, p, c]
// (U = symmetrised coupling rows [R, P], W = species weights [S, P, C], T rows of
// stride t_rows).  A warp owns one output row r and 32 channels; U[r, :] is a
// warp-uniform broadcast, W rows are coalesced over c.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) sc_fold_kernel(const float* __restrict__ U, const float* __restrict__ W,
                                                      float* __restrict__ T, int R, int P, int C, int64_t t_rows,
                                                      int64_t row0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  const int s = blockIdx.y;
  const int c = blockIdx.z * 32 + lane;
  if (r >= R || c >= C) return;
  const float* u = U + (int64_t)r * P;
  const float* w = W + (int64_t)s * P * C + c;
  float acc = 0.f;
  for (int p = 0; p < P; ++p) acc = fmaf(__ldg(u + p), __ldg(w + (int64_t)p * C), acc);
  T[((int64_t)s * t_rows + row0 + r) * C + c] = acc;
}

// Adjoint of the fold: dW[s, p, c] = sum_r U[r, p] dT[s, row0 + r, c].  One block per
// (p, s, 32 channels): its 8 warps take rows r = warp, warp + 8, ... and the partial
// sums meet in shared memory in a fixed order (deterministic, no atomics).
__global__ void __launch_bounds__(256) sc_fold_adjoint_kernel(const float* __restrict__ U,
                                                              const float* __restrict__ dT, float* __restrict__ dW,
                                                              int R, int P, int C, int64_t t_rows, int64_t row0) {
  __shared__ float part[8][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = blockIdx.x, s = blockIdx.y, c = blockIdx.z * 32 + lane;
  float acc = 0.f;
  if (c < C) {
    const float* g = dT + ((int64_t)s * t_rows + row0) * C + c;
    for (int r = warp; r < R; r += 8) acc = fmaf(__ldg(U + (int64_t)r * P + p), __ldg(g + (int64_t)r * C), acc);
  }
  part[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && c < C) {
    float total = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) total += part[k][lane];
    dW[((int64_t)s * P + p) * C + c] = total;
  }
}

}  // namespace ictc

using namespace ictc;

extern "C" int ictc_sc_fold(const float* usym, const float* weights, float* table, int rows, int cols,
                            int channels, int species, int64_t table_rows, int64_t row0, int adjoint, void* stream) {
  if (rows < 0 || cols < 0 || channels < 0 || species < 0 || row0 < 0 || row0 + rows > table_rows ||
      ((int64_t)rows * cols * channels * species > 0 && (!usym || !weights || !table))) {
    ictc_set_error("ictc_sc_fold: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  if ((int64_t)rows * cols * channels * species == 0) return ICTC_OK;
  const unsigned cz = (unsigned)((channels + 31) / 32);
  if (adjoint) {
    // weights <- dW [S, P, C]; table = dT [S, table_rows, C]
    sc_fold_adjoint_kernel<<<dim3((unsigned)cols, (unsigned)species, cz), 256, 0, (cudaStream_t)stream>>>(
        usym, table, const_cast<float*>(weights), rows, cols, channels, table_rows, row0);
  } else {
    sc_fold_kernel<<<dim3((unsigned)((rows + 7) / 8), (unsigned)species, cz), 256, 0, (cudaStream_t)stream>>>(
        usym, weights, table, rows, cols, channels, table_rows, row0);
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error("symmetric contraction fold launch failed: %s", cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}

extern "C" int64_t ictc_sc_table_rows(int lmax, int correlation, int target_lmax) {
  if (lmax < 0 || correlation < 1 || correlation > 3 || target_lmax < 0) return -1;
  const int D = (lmax + 1) * (lmax + 1);
  return (int64_t)sc_monomials(D, correlation) * (target_lmax + 1) * (target_lmax + 1);
}

extern "C" int ictc_sc_tile_nodes(void) { return kScNodes; }

static int sc_launch(bool backward, const float* x, const float* table, const int64_t* tiles,
                     const int32_t* tile_species, int64_t num_tiles, const float* grad_out, float* out,
                     float* grad_x, int channels, int lmax, int correlation, int target_lmax, void* stream) {
  if (num_tiles < 0 || channels <= 0 || target_lmax < 0 || target_lmax > lmax ||
      (num_tiles > 0 && (!x || !table || !tiles || !tile_species || (backward ? (!grad_out || !grad_x) : !out)))) {
    ictc_set_error("ictc_sc: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  SCFn fn = sc_kernel(lmax, correlation, backward);
  if (!fn) {
    ictc_set_error("ictc_sc: supported lmax 1..3 and correlation 1..3%s", "");
    return ICTC_ERR_UNSUPPORTED;
  }
  if (num_tiles == 0) return ICTC_OK;
  SCArgs a{};
  a.x = x; a.table = table; a.tiles = tiles; a.tile_species = tile_species; a.grad_out = grad_out; a.out = out;
  a.grad_x = grad_x; a.num_tiles = num_tiles; a.channels = channels; a.targets = target_lmax + 1;
  a.rows = ictc_sc_table_rows(lmax, correlation, target_lmax);
  int device = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int warps = sc_warps((lmax + 1) * (lmax + 1));
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, (const void*)fn, 32 * warps, 0);
  int64_t units = num_tiles * ((channels + 31) / 32);
  int64_t blocks = (units + warps - 1) / warps;
  int64_t cap = (int64_t)sms * (per_sm < 1 ? 1 : per_sm);
  fn<<<(int)(blocks < cap ? blocks : cap), 32 * warps, 0, (cudaStream_t)stream>>>(a);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error("symmetric contraction launch failed: %s", cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}

extern "C" int ictc_sc_forward(const float* x, const float* table, const int64_t* tiles, const int32_t* tile_species,
                               int64_t num_tiles, float* out, int channels, int lmax, int correlation,
                               int target_lmax, void* stream) {
  return sc_launch(false, x, table, tiles, tile_species, num_tiles, nullptr, out, nullptr, channels, lmax,
                   correlation, target_lmax, stream);
}

extern "C" int ictc_sc_backward(const float* x, const float* table, const int64_t* tiles,
                                const int32_t* tile_species, int64_t num_tiles, const float* grad_out,
                                float* grad_x, int channels, int lmax, int correlation, int target_lmax,
                                void* stream) {
  return sc_launch(true, x, table, tiles, tile_species, num_tiles, grad_out, nullptr, grad_x, channels, lmax,
                   correlation, target_lmax, stream);
}

static int sc_launch2(int kind, const float* x, const float* dir, const float* table, const int64_t* tiles,
                      const int32_t* tile_species, int64_t num_tiles, const float* grad_out, float* out,
                      float* grad_x, int channels, int lmax, int correlation, int target_lmax, void* stream) {
  if (num_tiles < 0 || channels <= 0 || target_lmax < 0 || target_lmax > lmax ||
      (num_tiles > 0 && (!x || !dir || !table || !tiles || !tile_species ||
                         (kind == 0 ? !out : (!grad_out || !grad_x))))) {
    ictc_set_error("ictc_sc second order: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  int warps = 1;
  SCFn fn = sc_kernel2(lmax, correlation, kind, &warps);
  if (!fn) {
    ictc_set_error("ictc_sc second order: supported lmax 1..3 and correlation 1..3%s", "");
    return ICTC_ERR_UNSUPPORTED;
  }
  if (num_tiles == 0) return ICTC_OK;
  SCArgs a{};
  a.x = x; a.dir = dir; a.table = table; a.tiles = tiles; a.tile_species = tile_species; a.grad_out = grad_out;
  a.out = out; a.grad_x = grad_x; a.num_tiles = num_tiles; a.channels = channels; a.targets = target_lmax + 1;
  a.rows = ictc_sc_table_rows(lmax, correlation, target_lmax);
  int device = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, (const void*)fn, 32 * warps, 0);
  const int64_t units = num_tiles * ((channels + 31) / 32);
  const int64_t blocks = (units + warps - 1) / warps;
  const int64_t cap = (int64_t)sms * (per_sm < 1 ? 1 : per_sm);
  fn<<<(int)(blocks < cap ? blocks : cap), 32 * warps, 0, (cudaStream_t)stream>>>(a);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error("symmetric contraction (second order) launch failed: %s", cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}

extern "C" int ictc_sc_directional(const float* x, const float* dir, const float* table, const int64_t* tiles,
                                   const int32_t* tile_species, int64_t num_tiles, float* out, int channels, int lmax,
                                   int correlation, int target_lmax, void* stream) {
  return sc_launch2(0, x, dir, table, tiles, tile_species, num_tiles, nullptr, out, nullptr, channels, lmax,
                    correlation, target_lmax, stream);
}

extern "C" int ictc_sc_hvp(const float* x, const float* dir, const float* table, const int64_t* tiles,
                           const int32_t* tile_species, int64_t num_tiles, const float* grad_out, float* grad_x,
                           int channels, int lmax, int correlation, int target_lmax, void* stream) {
  return sc_launch2(1, x, dir, table, tiles, tile_species, num_tiles, grad_out, nullptr, grad_x, channels, lmax,
                    correlation, target_lmax, stream);
}

extern "C" int ictc_sc_table_grad(const float* x, const float* dir, const float* grad_out, const int64_t* tiles,
                                  const int32_t* tile_species, int64_t num_tiles, float* grad_table, int species,
                                  int channels, int lmax, int correlation, int target_lmax, void* stream) {
  if (num_tiles < 0 || species < 1 || channels <= 0 || lmax < 1 || lmax > 3 || target_lmax < 0 ||
      target_lmax > lmax || correlation < 1 || correlation > 3 || !grad_table ||
      (num_tiles > 0 && (!x || !grad_out || !tiles || !tile_species))) {
    ictc_set_error("ictc_sc_table_grad: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  const int D = (lmax + 1) * (lmax + 1);
  const int mono = sc_monomials(D, correlation);
  SCGradArgs a{};
  a.x = x; a.dir = dir; a.grad_out = grad_out; a.tiles = tiles; a.tile_species = tile_species;
  a.grad_table = grad_table; a.num_tiles = num_tiles; a.rows_total = ictc_sc_table_rows(lmax, correlation, target_lmax);
  a.channels = channels; a.targets = target_lmax + 1; a.species = species; a.monomials = mono;
  int64_t row0 = 0, out_col = 0;
  for (int t = 0; t <= target_lmax; ++t) {
    const int M = 2 * t + 1;
    SCGradFn fn = sc_grad_kernel(lmax, correlation, M);
    if (!fn) {
      ictc_set_error("ictc_sc_table_grad: unsupported shape%s", "");
      return ICTC_ERR_UNSUPPORTED;
    }
    a.target = t; a.row0 = row0; a.out_col = out_col;
    const int rb = 64 / M;
    const int64_t units = (int64_t)species * ((channels + 31) / 32) * ((mono + rb - 1) / rb);
    fn<<<(unsigned)((units + 3) / 4), 128, 0, (cudaStream_t)stream>>>(a);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) {
      ictc_set_error("symmetric contraction table gradient launch failed: %s", cudaGetErrorString(err));
      return ICTC_ERR_CUDA;
    }
    row0 += (int64_t)mono * M;
    out_col += (int64_t)channels * M;
  }
  return ICTC_OK;
}
