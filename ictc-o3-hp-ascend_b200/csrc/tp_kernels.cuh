// Kernel templates of the path-preserving ICTC tensor product (standalone and graph message).
//
// Math (ictc_o3/basis/ictd_irreps.py:2669-2748, _project_group :2278-2283):
//   T(x, Y, g)[p, k, c] = g[p,c] w[p,c] sum_{i,j} x_{l1}[i,c] Y_{l2}[j] C_p[i,j,k]
// factored through bond[p,i,k] = sum_j Y[j] C_p[i,j,k] (the reference backend's
// bond projection, ictc_o3/backends/ascend/tensor_product.py:35-55).
// Graph message (ictc_o3/backends/ascend/tensor_product.py:189-218):
//   out[n] = sum_{e: dst_e = n} mask_e T(x[src_e], Y_e, g_e)
// evaluated node by node over a destination-sorted CSR, accumulating in
// registers (no atomics).  Its adjoint walks a source-sorted CSR so the
// feature gradient of a node is also a register accumulation.
#pragma once

#include "cg_pattern.h"
#include "tc_sm100.cuh"
#include "tp_device.cuh"

namespace ictc {

// bond_e[p, i, k] is identically zero when no harmonic component j couples (i, k)
// (28% of the (i, k) pairs up to l = 3); such entries are never formed.
template <int L1, int L2, int L3, int I, int K>
struct BondNonzero {
  static constexpr bool value = [] {
    for (int j = 0; j < 2 * L2 + 1; ++j)
      if (cg_nonzero(L1, L2, L3, I, j, K)) return true;
    return false;
  }();
};

// One bond entry of the message and adjoint kernels, formed in registers:
// sum_j C_p[i,j,k] Y_{l2}[j] over the structurally non-zero j, with the CG values
// read at compile-time offsets from the kernel's parameter bank (FFMA constant
// operands) and y = the edge's degree-l2 harmonics.
template <int L1, int L2, int L3, int CO, int I, int K, int CT>
__device__ __forceinline__ float bond_entry(const float (&coef)[CT], const float (&y)[2 * L2 + 1]) {
  constexpr int m2 = 2 * L2 + 1, m3 = 2 * L3 + 1;
  float b = 0.f;
  static_for<m2>([&](auto jc) {
    constexpr int j = decltype(jc)::value;
    if constexpr (CgNonzero<L1, L2, L3, I, j, K>::value) b = fmaf(coef[CO + (I * m3 + K) * m2 + j], y[j], b);
  });
  return b;
}

template <int L2>
__device__ __forceinline__ void load_harmonics(float (&y)[2 * L2 + 1], const float* s_y) {
#pragma unroll
  for (int j = 0; j < 2 * L2 + 1; ++j) y[j] = s_y[L2 * L2 + j];
}

// Column sums over a warp.  P = N rounded up to a power of two, S = log2(32 / P).
// On return lane L holds the total over the 32 lanes of column L >> S.  Each
// halving step keeps half of the live columns and trades the other half with the
// partner lane, so the N columns cost P - 1 + S shuffles instead of 5 N.
template <int N>
struct ColumnSum {
  static constexpr int P = N <= 1 ? 1 : N <= 2 ? 2 : N <= 4 ? 4 : N <= 8 ? 8 : N <= 16 ? 16 : 32;
  static constexpr int S = P == 1 ? 5 : P == 2 ? 4 : P == 4 ? 3 : P == 8 ? 2 : P == 16 ? 1 : 0;
};

template <int N>
__device__ __forceinline__ float warp_column_sum(const float (&v)[N], int lane) {
  static_assert(N <= 32, "at most 32 columns");
  constexpr int P = ColumnSum<N>::P;
  float w[P];
#pragma unroll
  for (int q = 0; q < P; ++q) w[q] = q < N ? v[q] : 0.f;
#pragma unroll
  for (int half = P / 2, off = 16; half >= 1; half >>= 1, off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int q = 0; q < half; ++q) {
      const float keep = upper ? w[q + half] : w[q];
      const float send = upper ? w[q] : w[q + half];
      w[q] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
#pragma unroll
  for (int off = (32 / P) >> 1; off > 0; off >>= 1) w[0] += __shfl_xor_sync(0xffffffffu, w[0], off);
  return w[0];
}

// ---------------------------------------------------------------------------
// Standalone forward: one warp per (instance, channel slice); every output
// block is written straight from registers with streaming stores.
// ---------------------------------------------------------------------------
template <int LI, int LE, int LO, int CPL, int LAYOUT>
__global__ void __launch_bounds__(kThreads) tp_forward_kernel(TPArgs a) {
  using PS = Paths<LI, LE, LO>;
  constexpr int A = PS::A, B = PS::B;
  extern __shared__ __align__(16) float smem[];
  float* s_coef = smem;
  int2* s_desc = reinterpret_cast<int2*>(smem + round4(PS::CT));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* s_y = smem + table_floats<PS>() + warp * warp_floats<PS>();
  float* s_bond = s_y + 32;
  load_tables<PS>(a, s_coef, s_desc);
  __syncthreads();

  const int C = a.channels;
  const int64_t items = a.rows * a.slices;
  for (int64_t item = (int64_t)blockIdx.x * kWarps + warp; item < items; item += (int64_t)gridDim.x * kWarps) {
    const int64_t e = item / a.slices;
    const int s = (int)(item - e * a.slices);
    const int c0 = (s * 32 + lane) * CPL;
    const bool active = c0 < C;
    if (lane < B) s_y[lane] = __ldg(a.harmonics + e * B + lane);
    __syncwarp();
    build_bond<PS>(s_coef, s_desc, s_y, s_bond, lane);
    __syncwarp();
    const float* xrow = a.features + e * A * C;
    float* orow = a.out + e * (int64_t)PS::ROWS * C;
    const float* grow = a.gates ? a.gates + e * (int64_t)PS::NP * C : nullptr;
    // Paths are ordered by input degree, so only one degree's rows are live at a time.
    static_for<LI + 1>([&](auto lc) {
      constexpr int l1 = decltype(lc)::value;
      constexpr int m1 = 2 * l1 + 1;
      float x[m1][CPL];
      load_degree<l1, CPL, LAYOUT>(x, xrow, C, c0, active, true);
      static_for<PS::NP>([&](auto pc) {
        constexpr int p = decltype(pc)::value;
        if constexpr (PS::T.l1[p] == decltype(lc)::value) {
          constexpr int m3 = 2 * PS::T.l3[p] + 1;
          constexpr int BO = PS::T.bond_off[p], RO = PS::T.out_row[p];
          float g[CPL];
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch) g[ch] = 1.f;
          if (active) {
            if (grow) load_vec_stream<CPL>(g, grow + p * C + c0);
            if (a.weight) {
              float w[CPL];
              load_vec<CPL>(w, a.weight + p * C + c0);
#pragma unroll
              for (int ch = 0; ch < CPL; ++ch) g[ch] *= w[ch];
            }
          }
#pragma unroll
          for (int k = 0; k < m3; ++k) {
            float acc[CPL];
#pragma unroll
            for (int ch = 0; ch < CPL; ++ch) acc[ch] = 0.f;
#pragma unroll
            for (int i = 0; i < m1; ++i) {
              const float b = s_bond[BO + i * m3 + k];
#pragma unroll
              for (int ch = 0; ch < CPL; ++ch) acc[ch] = fmaf(b, x[i][ch], acc[ch]);
            }
#pragma unroll
            for (int ch = 0; ch < CPL; ++ch) acc[ch] *= g[ch];
            if (active) {
              if constexpr (LAYOUT == kIrMul) {
                store_vec_stream<CPL>(orow + (int64_t)(RO + k) * C + c0, acc);
              } else {
#pragma unroll
                for (int ch = 0; ch < CPL; ++ch) __stcs(orow + (int64_t)RO * C + (c0 + ch) * m3 + k, acc[ch]);
              }
            }
          }
        }
      });
    });
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Graph-message forward over a destination CSR: one warp per (destination
// node, channel slice); the node's whole output row lives in registers.  Edge
// and source ids arrive in lane-parallel batches of 32.  Two ways to feed the
// edge loop:
//   * staged (one warp per node, rows in whole 16-byte units): a per-warp ring
//     of two shared buffers; the source row and gate row of edge k + 1 are
//     bulk-copied while edge k is computed (bounded mbarrier waits);
//   * direct: the next edge's source row, gate row and harmonics are loaded
//     into registers while the current edge is computed.
// ---------------------------------------------------------------------------
template <int LI, int LE, int LO, int CPL, int LAYOUT>
__global__ void __launch_bounds__(kThreads, (LO >= 3) ? 1 : 2)
    tp_message_forward_kernel(const __grid_constant__ CoefParams<Paths<LI, LE, LO>::CT> P) {
  using PS = Paths<LI, LE, LO>;
  constexpr int A = PS::A, B = PS::B, ROWS = PS::ROWS, NP = PS::NP;
  const TPArgs& a = P.a;
  extern __shared__ __align__(16) float smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* s_y = smem + table_floats<PS>() + warp * warp_floats<PS>();

  const int C = a.channels;
  const bool gate_bulk = bulk_rows(a.gates, NP * C * 4), x_bulk = bulk_rows(a.features, A * C * 4);
  const bool staged = a.stage_floats > 0;
  uint64_t* s_bar = nullptr;
  float* s_stage = nullptr;
  uint32_t phases = 0, turn = 0;
  if (staged) {
    char* base = reinterpret_cast<char*>(smem) + stage_offset_bytes((int)(smem_floats<PS>() * sizeof(float)));
    s_bar = reinterpret_cast<uint64_t*>(base) + 2 * warp;
    s_stage = reinterpret_cast<float*>(base + 128) + 2 * warp * a.stage_floats;
    if (lane == 0) {
      tc::mbar_init(s_bar, 1);
      tc::mbar_init(s_bar + 1, 1);
    }
    __syncwarp();
  }
  if constexpr (CPL > 1) {
    // Two channels per lane leave no registers for the direct path's pipeline:
    // the host launches this width only with staged rows.
    if (!staged) {
      if (threadIdx.x == 0 && a.status) atomicMax(a.status, 2);
      return;
    }
  }
  auto stage_issue = [&](int slot, int64_t e, int64_t xs) {
    if (lane == 0) {
      const uint32_t xbytes = A * C * 4, gbytes = a.gates ? NP * C * 4 : 0;
      float* buf = s_stage + slot * a.stage_floats;
      tc::mbar_arrive_expect(s_bar + slot, xbytes + gbytes);
      tc::bulk_load(buf, a.features + xs * (int64_t)A * C, xbytes, s_bar + slot);
      if (gbytes) tc::bulk_load(buf + A * C, a.gates + e * (int64_t)NP * C, gbytes, s_bar + slot);
    }
  };

  const int64_t items = a.rows * a.slices;
  for (int64_t item = (int64_t)blockIdx.x * kWarps + warp; item < items; item += (int64_t)gridDim.x * kWarps) {
    const int64_t n = item / a.slices;
    const int s = (int)(item - n * a.slices);
    const int c0 = (s * 32 + lane) * CPL;
    const bool active = c0 < C;
    float acc[ROWS][CPL];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int ch = 0; ch < CPL; ++ch) acc[r][ch] = 0.f;
    const int64_t k0 = a.offsets[n], k1 = a.offsets[n + 1];
    int64_t e_lane = 0, s_lane = 0;
    float m_lane = 1.f;
    int batch = 0;
    // Lane-parallel ids of the batch starting at edge k; the lane holding edge
    // k + kAheadL2 of the batch (edges 1..kAheadL2 at its start) pulls its gate
    // row and source row into L2.
    auto batch_ids = [&](int64_t k, int t) {
      if (t == 0) {
        const int64_t kl = k + lane;
        batch = (int)min((int64_t)32, k1 - k);
        if (kl < k1) {
          e_lane = a.order ? a.order[kl] : kl;
          s_lane = a.src[e_lane];
          m_lane = a.mask ? __ldg(a.mask + e_lane) : 1.f;
        }
      }
      if (s == 0 && (t == 0 ? (lane >= 1 && lane <= kAheadL2) : lane == t + kAheadL2) && lane < batch) {
        if (gate_bulk) prefetch_l2_bulk(a.gates + e_lane * (int64_t)NP * C, NP * C * 4);
        if (x_bulk) prefetch_l2_bulk(a.features + s_lane * (int64_t)A * C, A * C * 4);
      }
    };
    // acc += m T_p(x, Y, g) of one path p for one edge (g: the path's gate values).
    auto path_forward = [&](auto pc, const auto& x, const auto& gp, float m) {
      constexpr int p = decltype(pc)::value;
      constexpr int l1 = PS::T.l1[p], l2 = PS::T.l2[p], l3 = PS::T.l3[p];
      constexpr int m1 = 2 * l1 + 1, m3 = 2 * l3 + 1;
      constexpr int RO = PS::T.out_row[p], CO = PS::T.coef_off[p];
      float g[CPL];
#pragma unroll
      for (int ch = 0; ch < CPL; ++ch) g[ch] = gp[ch] * m;
      float y[2 * l2 + 1];
      load_harmonics<l2>(y, s_y);
      static_for<m3>([&](auto kc) {
        constexpr int kk = decltype(kc)::value;
        float base[CPL];
#pragma unroll
        for (int ch = 0; ch < CPL; ++ch) base[ch] = 0.f;
        static_for<m1>([&](auto ic) {
          constexpr int i = decltype(ic)::value;
          if constexpr (BondNonzero<l1, l2, l3, i, kk>::value) {
            const float b = bond_entry<l1, l2, l3, CO, i, kk>(P.coef, y);
#pragma unroll
            for (int ch = 0; ch < CPL; ++ch) base[ch] = fmaf(b, x[l1 * l1 + i][ch], base[ch]);
          }
        });
#pragma unroll
        for (int ch = 0; ch < CPL; ++ch) acc[RO + kk][ch] = fmaf(base[ch], g[ch], acc[RO + kk][ch]);
      });
    };

    if (staged) {
      bool pending = false;  // the copy of edge k is already in flight
      for (int64_t k = k0; k < k1; ++k) {
        const int t = (int)((k - k0) & 31);
        batch_ids(k, t);
        const int64_t e = __shfl_sync(0xffffffffu, e_lane, t);
        const int64_t xs = __shfl_sync(0xffffffffu, s_lane, t);
        const float m = __shfl_sync(0xffffffffu, m_lane, t);
        const int slot = (int)(turn & 1u);
        if (!pending) stage_issue(slot, e, xs);
        // The other buffer was released by the previous edge: start the next copy.
        pending = t + 1 < batch;
        if (pending) {
          const int64_t en = __shfl_sync(0xffffffffu, e_lane, t + 1);
          const int64_t sn = __shfl_sync(0xffffffffu, s_lane, t + 1);
          stage_issue(slot ^ 1, en, sn);
        }
        if (lane < B) s_y[lane] = __ldg(a.harmonics + e * B + lane);
        bool ok = tc::mbar_wait(s_bar + slot, (phases >> slot) & 1u, kStageWaitNs);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) {
          // Lost copy: record it, give the copies in flight a last bounded chance
          // to land (the buffers must not be written after the warp leaves), stop.
          // A drain that also times out means a copy may still write shared memory
          // after this CTA exits: status 3, which the host treats as fatal.
          if (lane == 0 && a.status) atomicMax(a.status, 1);
          bool drained = tc::mbar_wait(s_bar + slot, (phases >> slot) & 1u, kStageWaitNs);
          if (pending) drained = tc::mbar_wait(s_bar + (slot ^ 1), (phases >> (slot ^ 1)) & 1u, kStageWaitNs) && drained;
          if (!drained && lane == 0 && a.status) atomicMax(a.status, 3);
          return;
        }
        phases ^= 1u << slot;
        ++turn;
        __syncwarp();
        const float* buf = s_stage + slot * a.stage_floats;
        float x[A][CPL];
        load_features_shared<LI, CPL, LAYOUT>(x, buf, C, c0, active);
        const float* gbuf = buf + A * C;
        static_for<NP>([&](auto pc) {
          constexpr int p = decltype(pc)::value;
          float g[CPL];
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch) g[ch] = 1.f;
          if (a.gates && active) load_vec_shared<CPL>(g, gbuf + p * C + c0);
          path_forward(pc, x, g, m);
        });
        // Every staged value has been consumed (in-order issue): the buffer is free.
        __syncwarp();
      }
    } else if constexpr (CPL == 1) {
      // Registers of the edge being prefetched.
      float xn[A][CPL], gn[NP][CPL];
      float yn = 0.f, mn = 1.f;
      auto fetch = [&](int64_t k) {
        const int t = (int)((k - k0) & 31);
        batch_ids(k, t);
        const int64_t e = __shfl_sync(0xffffffffu, e_lane, t);
        const int64_t xs = __shfl_sync(0xffffffffu, s_lane, t);
        mn = __shfl_sync(0xffffffffu, m_lane, t);
        yn = lane < B ? __ldg(a.harmonics + e * B + lane) : 0.f;
        load_features<LI, CPL, LAYOUT>(xn, a.features + xs * A * C, C, c0, active, false);
        const float* grow = a.gates ? a.gates + e * (int64_t)NP * C : nullptr;
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          if (grow && active) load_vec_stream<CPL>(gn[p], grow + p * C + c0);
          else {
#pragma unroll
            for (int ch = 0; ch < CPL; ++ch) gn[p][ch] = 1.f;
          }
        }
      };
      if (k0 < k1) fetch(k0);
      for (int64_t k = k0; k < k1; ++k) {
        float x[A][CPL], g[NP][CPL];
#pragma unroll
        for (int r = 0; r < A; ++r)
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch) x[r][ch] = xn[r][ch];
        const float m = mn;
#pragma unroll
        for (int p = 0; p < NP; ++p)
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch) g[p][ch] = gn[p][ch];
        if (lane < B) s_y[lane] = yn;
        if (k + 1 < k1) fetch(k + 1);
        __syncwarp();
        static_for<NP>([&](auto pc) { path_forward(pc, x, g[decltype(pc)::value], m); });
        __syncwarp();
      }
    }
    if (active && a.weight) {
      // Path weights are constant over the edges: applied once per output block.
      static_for<NP>([&](auto pc) {
        constexpr int p = decltype(pc)::value;
        constexpr int m3 = 2 * PS::T.l3[p] + 1, RO = PS::T.out_row[p];
        float w[CPL];
        load_vec<CPL>(w, a.weight + p * C + c0);
#pragma unroll
        for (int kk = 0; kk < m3; ++kk)
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch) acc[RO + kk][ch] *= w[ch];
      });
    }
    if (active) {
      float* orow = a.out + n * (int64_t)ROWS * C;
      if constexpr (LAYOUT == kIrMul) {
#pragma unroll
        for (int r = 0; r < ROWS; ++r) store_vec<CPL>(orow + (int64_t)r * C + c0, acc[r]);
      } else {
        static_for<NP>([&](auto pc) {
          constexpr int p = decltype(pc)::value;
          constexpr int m3 = 2 * PS::T.l3[p] + 1;
          constexpr int RO = PS::T.out_row[p];
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch)
#pragma unroll
            for (int kk = 0; kk < m3; ++kk) orow[(int64_t)RO * C + (c0 + ch) * m3 + kk] = acc[RO + kk][ch];
        });
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Fused first-order adjoint, standalone (GRAPH = false: one "node" = one
// instance) or graph message over a source CSR (GRAPH = true).  For cotangent
// G of the output,
//   dx[node, l1, i, c] = sum_{e, p, k} bond_e[p,i,k] h_e[p,k,c]
//   dY[e, l2, j]       = sum_{p,i,k,c} C_p[i,j,k] x[i,c] h_e[p,k,c]
//   dgate[e, p, c]     = m_e w[p,c] sum_k G[p,k,c] sum_i bond_e[p,i,k] x[i,c]
// with h_e = m_e g_e w G[dst_e].  The `slices` warps of a node form a group
// that walks the same edges; their dY partials meet in shared memory behind a
// named barrier of the group (deterministic, no global atomics).
// ---------------------------------------------------------------------------
template <int LI, int LE, int LO, int CPL, int LAYOUT, bool GRAPH, bool STAGED = false>
__global__ void __launch_bounds__(kThreads, (GRAPH && LI >= 3) ? 1 : 2)
    tp_adjoint_kernel(const __grid_constant__ CoefParams<Paths<LI, LE, LO>::CT> P) {
  using PS = Paths<LI, LE, LO>;
  constexpr int A = PS::A, B = PS::B;
  const TPArgs& a = P.a;
  extern __shared__ __align__(16) float smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* s_y = smem + table_floats<PS>() + warp * warp_floats<PS>();
  float* s_bond = s_y + 32;
  float* s_dy = smem + table_floats<PS>() + kWarps * warp_floats<PS>();  // [kWarps][B]
  if constexpr (!GRAPH) {
    // Standalone: the warp builds each instance's bond row once in shared memory
    // (every entry is read by all its lanes; register-formed entries would raise
    // the register footprint of the l = 3 variant past its budget).
    load_tables<PS>(a, smem, reinterpret_cast<int2*>(smem + round4(PS::CT)));
    __syncthreads();
  }

  const int C = a.channels;
  const int slices = a.slices;
  const int groups = (int)(blockDim.x >> 5) / slices;
  const int group = warp / slices, s = warp - group * slices;
  const int c0 = (s * 32 + lane) * CPL;
  const bool active = c0 < C;
  const bool want_dx = a.grad_features != nullptr;
  const bool want_dy = a.grad_harmonics != nullptr;
  const bool want_dg = a.grad_gates != nullptr;

  // Adjoint of one path for one edge.  Rows XO + i of xl / dxl hold the path's
  // input degree and its gradient accumulators (XO = l1^2 for whole-row arrays,
  // 0 for one-degree arrays); dyp: this lane's partial dY of the edge.
  // Grow / grow point into this warp's shared staging buffer when `staged`.
  auto path_adjoint = [&](auto pc, auto xo, auto staged, auto& xl, auto& dxl, auto& dyp, const float* Grow,
                          const float* grow, float* dgrow, float m) {
    constexpr int p = decltype(pc)::value;
    constexpr int XO = decltype(xo)::value;
    constexpr int l1 = PS::T.l1[p], l2 = PS::T.l2[p], l3 = PS::T.l3[p];
    constexpr int m1 = 2 * l1 + 1, m2 = 2 * l2 + 1, m3 = 2 * l3 + 1;
    constexpr int RO = PS::T.out_row[p], CO = PS::T.coef_off[p];
    float G[m3][CPL];
    float gate[CPL], w[CPL];
#pragma unroll
    for (int ch = 0; ch < CPL; ++ch) { gate[ch] = 1.f; w[ch] = 1.f; }
    if (active) {
      if constexpr (decltype(staged)::value) {
        load_out_block_shared<CPL, LAYOUT, RO, m3>(G, Grow, C, c0);
        if (grow) load_vec_shared<CPL>(gate, grow + p * C + c0);
      } else {
        load_out_block<CPL, LAYOUT, RO, m3>(G, Grow, C, c0, !GRAPH);
        if (grow) load_vec_stream<CPL>(gate, grow + p * C + c0);
      }
      if (a.weight) load_vec<CPL>(w, a.weight + p * C + c0);
    } else {
#pragma unroll
      for (int kk = 0; kk < m3; ++kk)
#pragma unroll
        for (int ch = 0; ch < CPL; ++ch) G[kk][ch] = 0.f;
    }
    float h[m3][CPL], base[m3][CPL];
#pragma unroll
    for (int kk = 0; kk < m3; ++kk)
#pragma unroll
      for (int ch = 0; ch < CPL; ++ch) {
        h[kk][ch] = G[kk][ch] * (gate[ch] * w[ch] * m);
        base[kk][ch] = 0.f;
      }
    // Each bond entry (graph: formed in registers; standalone: read from the
    // instance's bond row) serves both the gate adjoint (base) and dx.
    constexpr int BO = PS::T.bond_off[p];
    (void)BO;
    float y[m2];
    if constexpr (GRAPH) load_harmonics<l2>(y, s_y);
    (void)y;
    static_for<m1>([&](auto ic) {
      constexpr int i = decltype(ic)::value;
      static_for<m3>([&](auto kc) {
        constexpr int kk = decltype(kc)::value;
        if constexpr (BondNonzero<l1, l2, l3, i, kk>::value) {
          float b;
          if constexpr (GRAPH) b = bond_entry<l1, l2, l3, CO, i, kk>(P.coef, y);
          else b = s_bond[BO + i * m3 + kk];
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch) {
            base[kk][ch] = fmaf(b, xl[XO + i][ch], base[kk][ch]);
            dxl[XO + i][ch] = fmaf(b, h[kk][ch], dxl[XO + i][ch]);
          }
        }
      });
    });
    if (want_dg) {
      float dg[CPL];
#pragma unroll
      for (int ch = 0; ch < CPL; ++ch) {
        float v = 0.f;
#pragma unroll
        for (int kk = 0; kk < m3; ++kk) v = fmaf(G[kk][ch], base[kk][ch], v);
        // d(effective gate) * d(effective gate)/d(gate): m w with gates, m without.
        dg[ch] = v * (grow ? m * w[ch] : m);
      }
      if (active) store_vec<CPL>(dgrow + p * C + c0, dg);
    }
    if (want_dy) {
      // dY_{l2}[j] += sum_{i,k} C_p[i,j,k] sum_c x[i,c] h[k,c]; structurally zero CG
      // terms are skipped at compile time, the values come from the parameter bank.
      static_for<m1>([&](auto ic) {
        constexpr int i = decltype(ic)::value;
        static_for<m3>([&](auto kc) {
          constexpr int kk = decltype(kc)::value;
          float t = 0.f;
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch) t = fmaf(xl[XO + i][ch], h[kk][ch], t);
          static_for<m2>([&](auto jc) {
            constexpr int j = decltype(jc)::value;
            if constexpr (CgNonzero<l1, l2, l3, i, j, kk>::value)
              dyp[l2 * l2 + j] = fmaf(P.coef[CO + (i * m3 + kk) * m2 + j], t, dyp[l2 * l2 + j]);
          });
        });
      });
    }
  };

  // dY of one edge: warp column sums, then a shared-memory sum over the group's slices.
  auto finish_dy = [&](auto& dyp, int64_t e) {
    constexpr int S = ColumnSum<B>::S;
    const float total = warp_column_sum<B>(dyp, lane);
    const int col = lane >> S;
    const bool owner = (lane & ((1 << S) - 1)) == 0 && col < B;
    if (slices == 1) {
      if (owner) a.grad_harmonics[e * B + col] = total;
    } else {
      if (owner) s_dy[warp * B + col] = total;
      group_barrier(1 + group, 32 * slices);
      if (s == 0 && lane < B) {
        float total = 0.f;
        for (int t = 0; t < slices; ++t) total += s_dy[(warp + t) * B + lane];
        a.grad_harmonics[e * B + lane] = total;
      }
      group_barrier(1 + group, 32 * slices);
    }
  };

  // Graph adjoint staging (one warp per node): each edge's output-gradient row and
  // gate row arrive in this warp's shared buffer by bulk copy, completed on its
  // mbarrier; the copy of the next edge is issued as soon as the buffer is free.
  constexpr bool staged = GRAPH && STAGED;
  if constexpr (staged) {
    // Launched only with a staging buffer (one warp per node, aligned rows).
    if (a.stage_floats <= 0 || a.slices != 1) {
      if (threadIdx.x == 0 && a.status) atomicMax(a.status, 2);
      return;
    }
  }
  uint64_t* s_bar = nullptr;
  float* s_stage = nullptr;
  uint32_t phase = 0;
  if (staged) {
    char* base = reinterpret_cast<char*>(smem) + stage_offset_bytes((int)(smem_floats<PS>() * sizeof(float)));
    s_bar = reinterpret_cast<uint64_t*>(base) + warp;
    s_stage = reinterpret_cast<float*>(base + 128) + warp * a.stage_floats;
    if (lane == 0) tc::mbar_init(s_bar, 1);
    __syncwarp();
  }
  auto stage_issue = [&](int64_t e, int64_t d) {
    if (lane == 0) {
      const uint32_t gbytes = PS::ROWS * C * 4, tbytes = a.gates ? PS::NP * C * 4 : 0;
      tc::mbar_arrive_expect(s_bar, gbytes + tbytes);
      tc::bulk_load(s_stage, a.grad_out + d * (int64_t)PS::ROWS * C, gbytes, s_bar);
      if (tbytes) tc::bulk_load(s_stage + PS::ROWS * C, a.gates + e * (int64_t)PS::NP * C, tbytes, s_bar);
    }
  };

  for (int64_t node = (int64_t)blockIdx.x * groups + group; node < a.rows; node += (int64_t)gridDim.x * groups) {
    if constexpr (!GRAPH) {
      // Standalone: one instance; paths are ordered by input degree, so one
      // degree's rows and gradients are live at a time.
      const int64_t e = node;
      if (lane < B) s_y[lane] = __ldg(a.harmonics + e * B + lane);
      __syncwarp();
      build_bond<PS>(smem, reinterpret_cast<const int2*>(smem + round4(PS::CT)), s_y, s_bond, lane);
      __syncwarp();
      float dyp[B];
#pragma unroll
      for (int j = 0; j < B; ++j) dyp[j] = 0.f;
      const float* Grow = a.grad_out + e * (int64_t)PS::ROWS * C;
      const float* grow = a.gates ? a.gates + e * (int64_t)PS::NP * C : nullptr;
      float* dgrow = want_dg ? a.grad_gates + e * (int64_t)PS::NP * C : nullptr;
      static_for<LI + 1>([&](auto lc) {
        constexpr int l1 = decltype(lc)::value;
        constexpr int m1 = 2 * l1 + 1;
        float xl[m1][CPL], dxl[m1][CPL];
        load_degree<l1, CPL, LAYOUT>(xl, a.features + e * A * C, C, c0, active, true);
#pragma unroll
        for (int i = 0; i < m1; ++i)
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch) dxl[i][ch] = 0.f;
        static_for<PS::NP>([&](auto pc) {
          if constexpr (PS::T.l1[decltype(pc)::value] == decltype(lc)::value)
            path_adjoint(pc, std::integral_constant<int, 0>{}, std::false_type{}, xl, dxl, dyp, Grow, grow, dgrow,
                         1.f);
        });
        if (want_dx && active) store_degree<l1, CPL, LAYOUT>(a.grad_features + e * A * C, dxl, C, c0);
      });
      if (want_dy) finish_dy(dyp, e);
      __syncwarp();
    } else {
      // Graph: a source node's rows stay in registers while its out-edges are walked.
      const bool gate_bulk = bulk_rows(a.gates, PS::NP * C * 4);
      const int64_t k0 = a.offsets[node], k1 = a.offsets[node + 1];
      float x[A][CPL], dx[A][CPL];
#pragma unroll
      for (int r = 0; r < A; ++r)
#pragma unroll
        for (int ch = 0; ch < CPL; ++ch) dx[r][ch] = 0.f;
      load_features<LI, CPL, LAYOUT>(x, a.features + node * A * C, C, c0, active, false);
      int64_t e_lane = 0, d_lane = 0;
      float m_lane = 1.f;
      int batch = 0;
      bool pending = false;  // staged: the copy of edge k is already in flight
      for (int64_t k = k0; k < k1; ++k) {
        const int t = (int)((k - k0) & 31);
        if (t == 0) {
          const int64_t kl = k + lane;
          batch = (int)min((int64_t)32, k1 - k);
          if (lane < batch) {
            e_lane = a.order ? a.order[kl] : kl;
            d_lane = a.dst[e_lane];
            m_lane = a.mask ? __ldg(a.mask + e_lane) : 1.f;
          }
        }
        // The lane holding edge k + kAheadL2 of this batch (edges 1..kAheadL2 at a
        // batch start) pulls its streamed gate row into L2.
        if (gate_bulk && s == 0 && (t == 0 ? (lane >= 1 && lane <= kAheadL2) : lane == t + kAheadL2) &&
            lane < batch)
          prefetch_l2_bulk(a.gates + e_lane * (int64_t)PS::NP * C, PS::NP * C * 4);
        const int64_t e = __shfl_sync(0xffffffffu, e_lane, t);
        const int64_t d = __shfl_sync(0xffffffffu, d_lane, t);
        const float m = __shfl_sync(0xffffffffu, m_lane, t);
        if constexpr (staged) {
          if (!pending) stage_issue(e, d);
          bool ok = tc::mbar_wait(s_bar, phase, kStageWaitNs);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) {
            // Lost copy: record it, give the copy in flight a last bounded chance to
            // land (the buffer must not be written after the warp leaves), and stop;
            // status 3 (fatal for the context) if that drain times out as well.
            if (lane == 0 && a.status) atomicMax(a.status, 1);
            const bool drained = tc::mbar_wait(s_bar, phase, kStageWaitNs);
            if (!drained && lane == 0 && a.status) atomicMax(a.status, 3);
            return;
          }
          phase ^= 1u;
        } else {
          // Pull the next edge's gathered output-gradient row and gate row into L1
          // while this edge computes; the group's slices split the lines.
          const int tn = t + 1 < batch ? t + 1 : t;
          const int64_t en = __shfl_sync(0xffffffffu, e_lane, tn);
          const int64_t dn = __shfl_sync(0xffffffffu, d_lane, tn);
          if (t + 1 < batch) {
            const char* grow_n = reinterpret_cast<const char*>(a.grad_out + dn * (int64_t)PS::ROWS * C);
            const int bytes = PS::ROWS * C * 4;
            for (int off = (s * 32 + lane) * 128; off < bytes; off += slices * 32 * 128) prefetch_l1(grow_n + off);
            if (a.gates) {
              const char* gate_n = reinterpret_cast<const char*>(a.gates + en * (int64_t)PS::NP * C);
              for (int off = (s * 32 + lane) * 128; off < PS::NP * C * 4; off += slices * 32 * 128)
                prefetch_l1(gate_n + off);
            }
          }
        }
        if (lane < B) s_y[lane] = __ldg(a.harmonics + e * B + lane);
        __syncwarp();
        float dyp[B];
#pragma unroll
        for (int j = 0; j < B; ++j) dyp[j] = 0.f;
        float* dgrow = want_dg ? a.grad_gates + e * (int64_t)PS::NP * C : nullptr;
        if constexpr (staged) {
          const float* grow = a.gates ? s_stage + PS::ROWS * C : nullptr;
          static_for<PS::NP>([&](auto pc) {
            constexpr int l1 = PS::T.l1[decltype(pc)::value];
            path_adjoint(pc, std::integral_constant<int, l1 * l1>{}, std::true_type{}, x, dx, dyp, s_stage, grow,
                         dgrow, m);
          });
          // Every staged value has been consumed (in-order issue): the buffer is free.
          __syncwarp();
          pending = k + 1 < k1 && t + 1 < batch;
          if (pending) {
            const int64_t en = __shfl_sync(0xffffffffu, e_lane, t + 1);
            const int64_t dn = __shfl_sync(0xffffffffu, d_lane, t + 1);
            stage_issue(en, dn);
          }
        } else {
          const float* Grow = a.grad_out + d * (int64_t)PS::ROWS * C;
          const float* grow = a.gates ? a.gates + e * (int64_t)PS::NP * C : nullptr;
          static_for<PS::NP>([&](auto pc) {
            constexpr int l1 = PS::T.l1[decltype(pc)::value];
            path_adjoint(pc, std::integral_constant<int, l1 * l1>{}, std::false_type{}, x, dx, dyp, Grow, grow,
                         dgrow, m);
          });
        }
        if (want_dy) finish_dy(dyp, e);
        __syncwarp();
      }
      if (want_dx && active) store_features<LI, CPL, LAYOUT>(a.grad_features + node * A * C, dx, C, c0);
    }
  }
}

// ---------------------------------------------------------------------------
// Variant registry (host side)
// ---------------------------------------------------------------------------
enum Kind : int { kForward = 0, kAdjoint = 1, kMessageForward = 2, kMessageAdjoint = 3, kKinds = 4 };

using Launcher = cudaError_t (*)(const TPArgs& args, const float* coef, int grid, int block, size_t smem,
                                 cudaStream_t stream);

struct Variant {
  int li, le, lo, cpl, layout, kind;
  const void* fn;       // kernel symbol (occupancy queries)
  Launcher launch;
  const void* fn_staged;  // graph adjoint with staged rows (null for other kinds)
  Launcher launch_staged;
  int np, bond_width, coef_total, rows, a, b;
  size_t smem;
};

template <class PS>
Variant describe(int cpl, int layout, int kind, int li, int le, int lo) {
  Variant v;
  v.li = li; v.le = le; v.lo = lo; v.cpl = cpl; v.layout = layout; v.kind = kind;
  v.np = PS::NP; v.bond_width = PS::BW; v.coef_total = PS::CT; v.rows = PS::ROWS; v.a = PS::A; v.b = PS::B;
  v.smem = sizeof(float) * smem_floats<PS>();
  return v;
}

template <int LI, int LE, int LO, int CPL, int LAYOUT, int KIND>
cudaError_t launch_plain(const TPArgs& args, const float*, int grid, int block, size_t smem, cudaStream_t stream) {
  tp_forward_kernel<LI, LE, LO, CPL, LAYOUT><<<grid, block, smem, stream>>>(args);
  return cudaGetLastError();
}

// Kernels that read the CG table from the parameter bank get it by value.
template <int LI, int LE, int LO, int CPL, int LAYOUT, int KIND, bool STAGED = false>
cudaError_t launch_coef(const TPArgs& args, const float* coef, int grid, int block, size_t smem,
                        cudaStream_t stream) {
  using PS = Paths<LI, LE, LO>;
  CoefParams<PS::CT> params;
  params.a = args;
  for (int t = 0; t < PS::CT; ++t) params.coef[t] = coef[t];
  if constexpr (KIND == kMessageForward)
    tp_message_forward_kernel<LI, LE, LO, CPL, LAYOUT><<<grid, block, smem, stream>>>(params);
  else
    tp_adjoint_kernel<LI, LE, LO, CPL, LAYOUT, KIND == kMessageAdjoint, STAGED><<<grid, block, smem, stream>>>(params);
  return cudaGetLastError();
}

template <int LI, int LE, int LO, int CPL, int LAYOUT, int KIND>
Variant make_variant() {
  using PS = Paths<LI, LE, LO>;
  Variant v = describe<PS>(CPL, LAYOUT, KIND, LI, LE, LO);
  v.fn_staged = nullptr;
  v.launch_staged = nullptr;
  if constexpr (KIND == kForward) {
    v.fn = (const void*)tp_forward_kernel<LI, LE, LO, CPL, LAYOUT>;
    v.launch = launch_plain<LI, LE, LO, CPL, LAYOUT, KIND>;
  } else if constexpr (KIND == kMessageForward) {
    v.fn = (const void*)tp_message_forward_kernel<LI, LE, LO, CPL, LAYOUT>;
    v.launch = launch_coef<LI, LE, LO, CPL, LAYOUT, KIND>;
  } else {
    v.fn = (const void*)tp_adjoint_kernel<LI, LE, LO, CPL, LAYOUT, KIND == kMessageAdjoint>;
    v.launch = launch_coef<LI, LE, LO, CPL, LAYOUT, KIND>;
    if constexpr (KIND == kMessageAdjoint && LO <= 2) {
      v.fn_staged = (const void*)tp_adjoint_kernel<LI, LE, LO, CPL, LAYOUT, true, true>;
      v.launch_staged = launch_coef<LI, LE, LO, CPL, LAYOUT, KIND, true>;
    }
  }
  return v;
}

}  // namespace ictc
