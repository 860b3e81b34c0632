// Channelwise path-preserving ICTC tensor product on sm_100a.
//
// Math (ictc_o3/basis/ictd_irreps.py:2669-2748 with _project_group :2278-2283):
//   out[e, p, k, c] = geff[e,p,c] * sum_{i,j} x_{l1}[e,i,c] Y_{l2}[e,j] C_p[i,j,k]
//   geff = gate[e,p,c] * w[p,c]        (either factor may be absent)
// Factored as bond[e,p,i,k] = sum_j Y[e,j] C_p[i,j,k] (the reference backend's
// "bond projection", ictc_o3/backends/ascend/tensor_product.py:35-55), then a
// per-channel (2l3+1)x(2l1+1) matrix-vector product.
//
// Work decomposition: one warp per (instance, channel slice).  A lane owns CPL
// consecutive channels, so every feature / gate / output row is read or written
// with one coalesced 32*CPL-float warp access (float4 at CPL=4).  The bond
// matrix of the instance (bond_width floats) is built cooperatively by the warp
// into shared memory from the dense CG table (also in shared memory) and then
// read as warp-uniform broadcasts.  Grids are persistent: a multiple of the SM
// count times the resident CTAs per SM.
#include "ictc_common.cuh"
#include "ictc_cuda.h"

#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

namespace ictc {

struct TPArgs {
  const float* __restrict__ features;
  const float* __restrict__ harmonics;
  const float* __restrict__ gates;
  const float* __restrict__ weight;
  const float* __restrict__ grad_out;
  float* __restrict__ out;
  float* __restrict__ grad_features;
  float* __restrict__ grad_harmonics;
  float* __restrict__ grad_gates;
  const float* __restrict__ coef;   // dense CG, [p][i][k][j]
  const int2* __restrict__ desc;    // per bond column: (yoff | m2 << 16, coef offset)
  int64_t rows;
  int channels;
  int slices;                       // channels / (32 * CPL)
};

constexpr int kWarps = 8;
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

template <int LI, int CPL, int LAYOUT>
__device__ __forceinline__ void load_features(float (&x)[(LI + 1) * (LI + 1)][CPL], const float* row,
                                              int channels, int c0) {
  if constexpr (LAYOUT == kIrMul) {
#pragma unroll
    for (int r = 0; r < (LI + 1) * (LI + 1); ++r) load_vec_stream<CPL>(x[r], row + (int64_t)r * channels + c0);
  } else {
    static_for<LI + 1>([&](auto lc) {
      constexpr int l = decltype(lc)::value;
      constexpr int m = 2 * l + 1;
      const float* blk = row + l * l * channels;
#pragma unroll
      for (int ch = 0; ch < CPL; ++ch)
#pragma unroll
        for (int i = 0; i < m; ++i) x[l * l + i][ch] = __ldg(blk + (c0 + ch) * m + i);
    });
  }
}

// ---------------------------------------------------------------------------
// Forward: out = TP(x, Y, geff)
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
    if (lane < B) s_y[lane] = __ldg(a.harmonics + e * B + lane);
    float x[A][CPL];
    load_features<LI, CPL, LAYOUT>(x, a.features + e * A * C, C, c0);
    __syncwarp();
    build_bond<PS>(s_coef, s_desc, s_y, s_bond, lane);
    __syncwarp();
    float* orow = a.out + e * (int64_t)PS::ROWS * C;
    const float* grow = a.gates ? a.gates + e * (int64_t)PS::NP * C : nullptr;
    static_for<PS::NP>([&](auto pc) {
      constexpr int p = decltype(pc)::value;
      constexpr int l1 = PS::T.l1[p], l3 = PS::T.l3[p];
      constexpr int m1 = 2 * l1 + 1, m3 = 2 * l3 + 1;
      constexpr int BO = PS::T.bond_off[p], RO = PS::T.out_row[p];
      float g[CPL];
#pragma unroll
      for (int ch = 0; ch < CPL; ++ch) g[ch] = 1.f;
      if (grow) load_vec_stream<CPL>(g, grow + p * C + c0);
      if (a.weight) {
        float w[CPL];
        load_vec<CPL>(w, a.weight + p * C + c0);
#pragma unroll
        for (int ch = 0; ch < CPL; ++ch) g[ch] *= w[ch];
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
          for (int ch = 0; ch < CPL; ++ch) acc[ch] = fmaf(b, x[l1 * l1 + i][ch], acc[ch]);
        }
#pragma unroll
        for (int ch = 0; ch < CPL; ++ch) acc[ch] *= g[ch];
        if constexpr (LAYOUT == kIrMul) {
          store_vec_stream<CPL>(orow + (int64_t)(RO + k) * C + c0, acc);
        } else {
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch) __stcs(orow + (int64_t)RO * C + (c0 + ch) * m3 + k, acc[ch]);
        }
      }
    });
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Fused first-order adjoint: given G = d(loss)/d(out),
//   dx[e,l1,i,c] += sum_{p,k} bond[p,i,k] geff[p,c] G[p,k,c]
//   dY[e,l2,j]   += sum_{p,i,k,c} C_p[i,j,k] x[i,c] geff[p,c] G[p,k,c]
//   dgate[e,p,c]  = w[p,c] sum_k G[p,k,c] sum_i bond[p,i,k] x[i,c]
// One CTA iteration covers kWarps / slices instances; the slices of one
// instance sit in one CTA and their dY partials are summed in shared memory
// (deterministic, no global atomics).
// ---------------------------------------------------------------------------
template <int LI, int LE, int LO, int CPL, int LAYOUT>
__global__ void __launch_bounds__(kThreads) tp_backward_kernel(TPArgs a) {
  using PS = Paths<LI, LE, LO>;
  constexpr int A = PS::A, B = PS::B;
  extern __shared__ __align__(16) float smem[];
  float* s_coef = smem;
  int2* s_desc = reinterpret_cast<int2*>(smem + round4(PS::CT));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* s_y = smem + table_floats<PS>() + warp * warp_floats<PS>();
  float* s_bond = s_y + 32;
  float* s_dy = smem + table_floats<PS>() + kWarps * warp_floats<PS>();  // [kWarps][B]
  load_tables<PS>(a, s_coef, s_desc);
  __syncthreads();

  const int C = a.channels;
  const int per_cta = kWarps / a.slices;
  const int el = warp / a.slices, s = warp - el * a.slices;
  const int c0 = (s * 32 + lane) * CPL;
  const bool want_dx = a.grad_features != nullptr;
  const bool want_dy = a.grad_harmonics != nullptr;
  const bool want_dg = a.grad_gates != nullptr;
  for (int64_t first = (int64_t)blockIdx.x * per_cta; first < a.rows; first += (int64_t)gridDim.x * per_cta) {
    const int64_t e = first + el;
    const bool valid = el < per_cta && e < a.rows;
    float dyp[B];
#pragma unroll
    for (int j = 0; j < B; ++j) dyp[j] = 0.f;
    if (valid) {
      if (lane < B) s_y[lane] = __ldg(a.harmonics + e * B + lane);
      float x[A][CPL];
      float dx[A][CPL];
#pragma unroll
      for (int r = 0; r < A; ++r)
#pragma unroll
        for (int ch = 0; ch < CPL; ++ch) dx[r][ch] = 0.f;
      load_features<LI, CPL, LAYOUT>(x, a.features + e * A * C, C, c0);
      __syncwarp();
      build_bond<PS>(s_coef, s_desc, s_y, s_bond, lane);
      __syncwarp();
      const float* Grow = a.grad_out + e * (int64_t)PS::ROWS * C;
      const float* grow = a.gates ? a.gates + e * (int64_t)PS::NP * C : nullptr;
      float* dgrow = want_dg ? a.grad_gates + e * (int64_t)PS::NP * C : nullptr;
      static_for<PS::NP>([&](auto pc) {
        constexpr int p = decltype(pc)::value;
        constexpr int l1 = PS::T.l1[p], l2 = PS::T.l2[p], l3 = PS::T.l3[p];
        constexpr int m1 = 2 * l1 + 1, m2 = 2 * l2 + 1, m3 = 2 * l3 + 1;
        constexpr int BO = PS::T.bond_off[p], RO = PS::T.out_row[p], CO = PS::T.coef_off[p];
        float G[m3][CPL];
        if constexpr (LAYOUT == kIrMul) {
#pragma unroll
          for (int k = 0; k < m3; ++k) load_vec_stream<CPL>(G[k], Grow + (int64_t)(RO + k) * C + c0);
        } else {
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch)
#pragma unroll
            for (int k = 0; k < m3; ++k) G[k][ch] = __ldcs(Grow + (int64_t)RO * C + (c0 + ch) * m3 + k);
        }
        float gate[CPL], w[CPL];
#pragma unroll
        for (int ch = 0; ch < CPL; ++ch) { gate[ch] = 1.f; w[ch] = 1.f; }
        if (grow) load_vec_stream<CPL>(gate, grow + p * C + c0);
        if (a.weight) load_vec<CPL>(w, a.weight + p * C + c0);
        if (want_dg) {
          float dg[CPL];
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch) dg[ch] = 0.f;
#pragma unroll
          for (int k = 0; k < m3; ++k) {
#pragma unroll
            for (int ch = 0; ch < CPL; ++ch) {
              float base = 0.f;
#pragma unroll
              for (int i = 0; i < m1; ++i) base = fmaf(s_bond[BO + i * m3 + k], x[l1 * l1 + i][ch], base);
              dg[ch] = fmaf(G[k][ch], base, dg[ch]);
            }
          }
          // d(geff) * d(geff)/d(gate): w when gates are given; per-instance weight grad otherwise.
          if (grow) {
#pragma unroll
            for (int ch = 0; ch < CPL; ++ch) dg[ch] *= w[ch];
          }
          store_vec<CPL>(dgrow + p * C + c0, dg);
        }
        float h[m3][CPL];
#pragma unroll
        for (int k = 0; k < m3; ++k)
#pragma unroll
          for (int ch = 0; ch < CPL; ++ch) h[k][ch] = G[k][ch] * (gate[ch] * w[ch]);
        if (want_dx) {
#pragma unroll
          for (int i = 0; i < m1; ++i)
#pragma unroll
            for (int k = 0; k < m3; ++k) {
              const float b = s_bond[BO + i * m3 + k];
#pragma unroll
              for (int ch = 0; ch < CPL; ++ch) dx[l1 * l1 + i][ch] = fmaf(b, h[k][ch], dx[l1 * l1 + i][ch]);
            }
        }
        if (want_dy) {
#pragma unroll
          for (int i = 0; i < m1; ++i)
#pragma unroll
            for (int k = 0; k < m3; ++k) {
              float t = 0.f;
#pragma unroll
              for (int ch = 0; ch < CPL; ++ch) t = fmaf(x[l1 * l1 + i][ch], h[k][ch], t);
#pragma unroll
              for (int j = 0; j < m2; ++j)
                dyp[l2 * l2 + j] = fmaf(s_coef[CO + (i * m3 + k) * m2 + j], t, dyp[l2 * l2 + j]);
            }
        }
      });
      if (want_dx) {
        float* dxrow = a.grad_features + e * A * C;
        if constexpr (LAYOUT == kIrMul) {
#pragma unroll
          for (int r = 0; r < A; ++r) store_vec<CPL>(dxrow + (int64_t)r * C + c0, dx[r]);
        } else {
          static_for<LI + 1>([&](auto lc) {
            constexpr int l = decltype(lc)::value;
            constexpr int m = 2 * l + 1;
#pragma unroll
            for (int ch = 0; ch < CPL; ++ch)
#pragma unroll
              for (int i = 0; i < m; ++i) dxrow[l * l * C + (c0 + ch) * m + i] = dx[l * l + i][ch];
          });
        }
      }
    }
    if (want_dy) {
      // Warp all-reduce of the per-lane partials, then a shared-memory sum over slices.
      float mine = 0.f;
#pragma unroll
      for (int j = 0; j < B; ++j) {
        float v = dyp[j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == j) mine = v;
      }
      if (lane < B) s_dy[warp * B + lane] = mine;
      __syncthreads();
      if (valid && s == 0 && lane < B) {
        float total = 0.f;
        for (int t = 0; t < a.slices; ++t) total += s_dy[(warp + t) * B + lane];
        a.grad_harmonics[e * B + lane] = total;
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------
// Host side: plans, dispatch, launch configuration.
// ---------------------------------------------------------------------------

using KernelFn = void (*)(TPArgs);

struct Variant {
  int li, le, lo, cpl, layout;
  KernelFn fwd, bwd;
  int np, bond_width, coef_total, rows, a, b;
  size_t smem_fwd, smem_bwd;
};

template <int LI, int LE, int LO, int CPL, int LAYOUT>
Variant make_variant() {
  using PS = Paths<LI, LE, LO>;
  Variant v;
  v.li = LI; v.le = LE; v.lo = LO; v.cpl = CPL; v.layout = LAYOUT;
  v.fwd = tp_forward_kernel<LI, LE, LO, CPL, LAYOUT>;
  v.bwd = tp_backward_kernel<LI, LE, LO, CPL, LAYOUT>;
  v.np = PS::NP; v.bond_width = PS::BW; v.coef_total = PS::CT; v.rows = PS::ROWS; v.a = PS::A; v.b = PS::B;
  v.smem_fwd = sizeof(float) * (table_floats<PS>() + kWarps * warp_floats<PS>());
  v.smem_bwd = v.smem_fwd + sizeof(float) * kWarps * PS::B;
  return v;
}

#define ICTC_TP_LAYOUTS(LI, LE, LO, CPL) \
  make_variant<LI, LE, LO, CPL, kIrMul>(), make_variant<LI, LE, LO, CPL, kMulIr>()
#define ICTC_TP_CPLS(LI, LE, LO) \
  ICTC_TP_LAYOUTS(LI, LE, LO, 1), ICTC_TP_LAYOUTS(LI, LE, LO, 2), ICTC_TP_LAYOUTS(LI, LE, LO, 4)

static const std::vector<Variant>& variants() {
  static const std::vector<Variant> table = {
      ICTC_TP_CPLS(0, 1, 1), ICTC_TP_CPLS(1, 1, 1),
      ICTC_TP_CPLS(0, 2, 2), ICTC_TP_CPLS(2, 2, 2),
      ICTC_TP_CPLS(0, 3, 3), ICTC_TP_CPLS(3, 3, 3),
  };
  return table;
}

}  // namespace ictc

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
using namespace ictc;

struct ictc_tp_plan {
  int channels, li, le, lo, layout;
  int cpl_fwd, cpl_bwd;
  const Variant* fwd;
  const Variant* bwd;
  float* d_coef;
  int2* d_desc;
  int device;
  int grid_fwd, grid_bwd;
};

static thread_local char g_error[512] = "";

void ictc_set_error(const char* fmt, const char* detail) {
  snprintf(g_error, sizeof(g_error), fmt, detail ? detail : "");
}

extern "C" const char* ictc_last_error(void) { return g_error; }

extern "C" int ictc_version(void) { return ICTC_ABI_VERSION; }

static const Variant* find_variant(int li, int le, int lo, int cpl, int layout) {
  for (const Variant& v : variants())
    if (v.li == li && v.le == le && v.lo == lo && v.cpl == cpl && v.layout == layout) return &v;
  return nullptr;
}

static int pick_cpl(int channels, int preferred) {
  for (int cpl = preferred; cpl >= 1; cpl /= 2)
    if (channels % (32 * cpl) == 0 && (channels / (32 * cpl)) <= kWarps && (kWarps % (channels / (32 * cpl))) == 0)
      return cpl;
  return 0;
}

static int grid_for(KernelFn fn, size_t smem, int device) {
  int sms = 0, per_sm = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, smem);
  if (per_sm < 1) per_sm = 1;
  return sms * per_sm;
}

extern "C" int ictc_tp_plan_create(int channels, int input_lmax, int edge_lmax, int output_lmax, int layout,
                                   int num_paths, const int32_t* paths, const double* cg, int64_t cg_len,
                                   int cpl_forward, int cpl_backward, ictc_tp_plan** out) {
  if (!out || !paths || !cg) {
    ictc_set_error("ictc_tp_plan_create: null argument%s", "");
    return ICTC_ERR_INVALID;
  }
  *out = nullptr;
  if (layout != kIrMul && layout != kMulIr) {
    ictc_set_error("ictc_tp_plan_create: layout must be 0 (ir_mul) or 1 (mul_ir)%s", "");
    return ICTC_ERR_INVALID;
  }
  int cf = pick_cpl(channels, cpl_forward > 0 ? cpl_forward : 4);
  int cb = pick_cpl(channels, cpl_backward > 0 ? cpl_backward : 2);
  if (channels <= 0 || cf == 0 || cb == 0) {
    ictc_set_error("ictc_tp_plan_create: channels must be a positive multiple of 32 and at most 256%s", "");
    return ICTC_ERR_UNSUPPORTED;
  }
  const Variant* vf = find_variant(input_lmax, edge_lmax, output_lmax, cf, layout);
  const Variant* vb = find_variant(input_lmax, edge_lmax, output_lmax, cb, layout);
  if (!vf || !vb) {
    ictc_set_error("ictc_tp_plan_create: no kernel for this (input_lmax, edge_lmax, output_lmax)%s", "");
    return ICTC_ERR_UNSUPPORTED;
  }
  const PathTable ref = make_paths(input_lmax, edge_lmax, output_lmax);
  if (num_paths != vf->np) {
    ictc_set_error("ictc_tp_plan_create: path list does not match the operator path set%s", "");
    return ICTC_ERR_UNSUPPORTED;
  }
  int64_t expect = 0;
  for (int p = 0; p < num_paths; ++p) {
    if (paths[3 * p] != ref.l1[p] || paths[3 * p + 1] != ref.l2[p] || paths[3 * p + 2] != ref.l3[p]) {
      ictc_set_error("ictc_tp_plan_create: path order differs from the operator path order%s", "");
      return ICTC_ERR_UNSUPPORTED;
    }
    expect += (2 * ref.l1[p] + 1) * (2 * ref.l2[p] + 1) * (2 * ref.l3[p] + 1);
  }
  if (cg_len != expect) {
    ictc_set_error("ictc_tp_plan_create: CG buffer length mismatch%s", "");
    return ICTC_ERR_INVALID;
  }
  // Re-lay the per-path CG tensors C_p[i][j][k] as [p][i][k][j] and build the
  // bond column descriptors.
  std::vector<float> coef(ref.coef_total);
  std::vector<int2> desc(ref.bond_width);
  int64_t src = 0;
  for (int p = 0; p < num_paths; ++p) {
    int m1 = 2 * ref.l1[p] + 1, m2 = 2 * ref.l2[p] + 1, m3 = 2 * ref.l3[p] + 1;
    for (int i = 0; i < m1; ++i)
      for (int j = 0; j < m2; ++j)
        for (int k = 0; k < m3; ++k)
          coef[ref.coef_off[p] + (i * m3 + k) * m2 + j] = (float)cg[src + (i * m2 + j) * m3 + k];
    for (int i = 0; i < m1; ++i)
      for (int k = 0; k < m3; ++k) {
        int col = ref.bond_off[p] + i * m3 + k;
        desc[col].x = (ref.l2[p] * ref.l2[p]) | (m2 << 16);
        desc[col].y = ref.coef_off[p] + (i * m3 + k) * m2;
      }
    src += (int64_t)m1 * m2 * m3;
  }
  ictc_tp_plan* plan = new (std::nothrow) ictc_tp_plan();
  if (!plan) return ICTC_ERR_NOMEM;
  plan->channels = channels; plan->li = input_lmax; plan->le = edge_lmax; plan->lo = output_lmax;
  plan->layout = layout; plan->cpl_fwd = cf; plan->cpl_bwd = cb; plan->fwd = vf; plan->bwd = vb;
  cudaGetDevice(&plan->device);
  if (cudaMalloc(&plan->d_coef, sizeof(float) * (coef.size() + 4)) != cudaSuccess ||
      cudaMalloc(&plan->d_desc, sizeof(int2) * (desc.size() + 4)) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(plan->d_coef);
    delete plan;
    ictc_set_error("ictc_tp_plan_create: device allocation failed%s", "");
    return ICTC_ERR_NOMEM;
  }
  cudaMemcpy(plan->d_coef, coef.data(), sizeof(float) * coef.size(), cudaMemcpyHostToDevice);
  cudaMemcpy(plan->d_desc, desc.data(), sizeof(int2) * desc.size(), cudaMemcpyHostToDevice);
  plan->grid_fwd = grid_for(vf->fwd, vf->smem_fwd, plan->device);
  plan->grid_bwd = grid_for(vb->bwd, vb->smem_bwd, plan->device);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error("ictc_tp_plan_create: %s", cudaGetErrorString(err));
    cudaFree(plan->d_coef);
    cudaFree(plan->d_desc);
    delete plan;
    return ICTC_ERR_CUDA;
  }
  *out = plan;
  return ICTC_OK;
}

extern "C" int ictc_tp_plan_destroy(ictc_tp_plan* plan) {
  if (!plan) return ICTC_OK;
  cudaFree(plan->d_coef);
  cudaFree(plan->d_desc);
  delete plan;
  return ICTC_OK;
}

extern "C" int ictc_tp_plan_info(const ictc_tp_plan* plan, int64_t* info, int n) {
  if (!plan || !info) return ICTC_ERR_INVALID;
  int64_t values[8] = {plan->fwd->np, plan->fwd->bond_width, plan->fwd->rows * (int64_t)plan->channels,
                       plan->fwd->a * (int64_t)plan->channels, plan->fwd->b, plan->cpl_fwd, plan->cpl_bwd,
                       plan->grid_fwd};
  for (int t = 0; t < n && t < 8; ++t) info[t] = values[t];
  return ICTC_OK;
}

static int launch(KernelFn fn, int grid_cap, size_t smem, int64_t work_blocks, const TPArgs& args,
                  void* stream) {
  if (work_blocks <= 0) return ICTC_OK;
  int grid = (int)(work_blocks < grid_cap ? work_blocks : grid_cap);
  fn<<<grid, kThreads, smem, (cudaStream_t)stream>>>(args);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error("tensor-product launch failed: %s", cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}

extern "C" int ictc_tp_forward(const ictc_tp_plan* plan, const float* features, const float* harmonics,
                               const float* gates, const float* weight, float* out, int64_t rows,
                               void* stream) {
  if (!plan || rows < 0 || (rows > 0 && (!features || !harmonics || !out))) {
    ictc_set_error("ictc_tp_forward: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  TPArgs a{};
  a.features = features; a.harmonics = harmonics; a.gates = gates; a.weight = weight; a.out = out;
  a.coef = plan->d_coef; a.desc = plan->d_desc; a.rows = rows; a.channels = plan->channels;
  a.slices = plan->channels / (32 * plan->cpl_fwd);
  int64_t items = rows * a.slices;
  return launch(plan->fwd->fwd, plan->grid_fwd, plan->fwd->smem_fwd, (items + kWarps - 1) / kWarps, a, stream);
}

extern "C" int ictc_tp_backward(const ictc_tp_plan* plan, const float* features, const float* harmonics,
                                const float* gates, const float* weight, const float* grad_out,
                                float* grad_features, float* grad_harmonics, float* grad_gates, int64_t rows,
                                void* stream) {
  if (!plan || rows < 0 || (rows > 0 && (!features || !harmonics || !grad_out))) {
    ictc_set_error("ictc_tp_backward: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  TPArgs a{};
  a.features = features; a.harmonics = harmonics; a.gates = gates; a.weight = weight; a.grad_out = grad_out;
  a.grad_features = grad_features; a.grad_harmonics = grad_harmonics; a.grad_gates = grad_gates;
  a.coef = plan->d_coef; a.desc = plan->d_desc; a.rows = rows; a.channels = plan->channels;
  a.slices = plan->channels / (32 * plan->cpl_bwd);
  int per_cta = kWarps / a.slices;
  return launch(plan->bwd->bwd, plan->grid_bwd, plan->bwd->smem_bwd, (rows + per_cta - 1) / per_cta, a, stream);
}
