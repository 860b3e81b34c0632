// ICTC direction harmonics Y_l(n), l = 0..LMAX, and their derivatives.
//
// Y_l(n)[m] = sum_d n_x^a n_y^b n_z^c H_l[d, m], (a, b, c) running over the
// degree-l monomials in ICTC order (a outer, b inner, c = l - a - b), with
// H_l = multinomial * (G_l B_l) * component scale precomputed on the host
// (ictc_o3/basis/ictd_irreps.py:1113-1168, _dir_proj_cpu_f64 :913-923,
// _direction_component_scale_cpu_f64 :926-953).  Modes:
//   0  forward:  Y = f(n)
//   1  adjoint:  dn = J(n)^T gY
//   2  second order of mode 1 for a cotangent hn of dn:
//        d_gY = J(n) hn            d_n = sum_m gY[m] H(n)[m] hn
// One thread per row; the monomial table lives in shared memory.
#include "ictc_common.cuh"
#include "ictc_cuda.h"

#include <cstdio>

void ictc_set_error(const char* fmt, const char* detail);

namespace ictc {

constexpr int kHarmThreads = 256;

template <int LMAX>
__host__ __device__ constexpr int harmonic_table_size() {
  int total = 0;
  for (int l = 1; l <= LMAX; ++l) total += (l + 1) * (l + 2) / 2 * (2 * l + 1);
  return total;
}

template <int LMAX>
__global__ void __launch_bounds__(kHarmThreads) harmonics_kernel(const float* __restrict__ n,
                                                                 const float* __restrict__ table,
                                                                 const float* __restrict__ gy,
                                                                 const float* __restrict__ hn,
                                                                 float* __restrict__ out0,
                                                                 float* __restrict__ out1, int64_t rows,
                                                                 int mode) {
  constexpr int W = (LMAX + 1) * (LMAX + 1);
  constexpr int T = harmonic_table_size<LMAX>();
  __shared__ float s_table[T > 0 ? T : 1];
  for (int t = threadIdx.x; t < T; t += blockDim.x) s_table[t] = table[t];
  __syncthreads();
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < rows; e += (int64_t)gridDim.x * blockDim.x) {
    const float v[3] = {n[3 * e], n[3 * e + 1], n[3 * e + 2]};
    float pw[3][LMAX + 1];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      pw[c][0] = 1.f;
#pragma unroll
      for (int k = 1; k <= LMAX; ++k) pw[c][k] = pw[c][k - 1] * v[c];
    }
    float g[W], h3[3];
    if (mode >= 1) {
#pragma unroll
      for (int m = 0; m < W; ++m) g[m] = gy[e * W + m];
    }
    if (mode == 2) {
#pragma unroll
      for (int c = 0; c < 3; ++c) h3[c] = hn[3 * e + c];
    }
    float dn[3] = {0.f, 0.f, 0.f};
    if (mode == 0) out0[e * W] = 1.f;
    if (mode == 2) out0[e * W] = 0.f;
    int toff = 0;
#pragma unroll
    for (int l = 1; l <= LMAX; ++l) {
      constexpr int dummy = 0;
      (void)dummy;
      const int m_count = 2 * l + 1;
      float y[2 * LMAX + 1];
#pragma unroll
      for (int m = 0; m < 2 * LMAX + 1; ++m) y[m] = 0.f;
      int d = 0;
#pragma unroll
      for (int a = 0; a <= l; ++a) {
#pragma unroll
        for (int b = 0; b <= l - a; ++b, ++d) {
          const int c = l - a - b;
          const float* row = s_table + toff + d * m_count;
          if (mode == 0) {
            const float mono = pw[0][a] * pw[1][b] * pw[2][c];
#pragma unroll
            for (int m = 0; m < 2 * LMAX + 1; ++m)
              if (m < m_count) y[m] = fmaf(mono, row[m], y[m]);
          } else {
            // s = sum_m gY[m] H[d, m]: the weight of this monomial in <gY, Y>.
            float s = 0.f;
            float jv = 0.f;  // directional derivative of the monomial along hn (mode 2)
            const float gx = a ? a * pw[0][a - 1] * pw[1][b] * pw[2][c] : 0.f;
            const float gyv = b ? b * pw[0][a] * pw[1][b - 1] * pw[2][c] : 0.f;
            const float gz = c ? c * pw[0][a] * pw[1][b] * pw[2][c - 1] : 0.f;
#pragma unroll
            for (int m = 0; m < 2 * LMAX + 1; ++m)
              if (m < m_count) s = fmaf(g[l * l + m], row[m], s);
            if (mode == 1) {
              dn[0] = fmaf(s, gx, dn[0]);
              dn[1] = fmaf(s, gyv, dn[1]);
              dn[2] = fmaf(s, gz, dn[2]);
            } else {
              jv = gx * h3[0] + gyv * h3[1] + gz * h3[2];
#pragma unroll
              for (int m = 0; m < 2 * LMAX + 1; ++m)
                if (m < m_count) y[m] = fmaf(jv, row[m], y[m]);
              // Hessian of the monomial applied to hn.
              const float hxx = a >= 2 ? a * (a - 1) * pw[0][a >= 2 ? a - 2 : 0] * pw[1][b] * pw[2][c] : 0.f;
              const float hyy = b >= 2 ? b * (b - 1) * pw[0][a] * pw[1][b >= 2 ? b - 2 : 0] * pw[2][c] : 0.f;
              const float hzz = c >= 2 ? c * (c - 1) * pw[0][a] * pw[1][b] * pw[2][c >= 2 ? c - 2 : 0] : 0.f;
              const float hxy = (a && b) ? a * b * pw[0][a ? a - 1 : 0] * pw[1][b ? b - 1 : 0] * pw[2][c] : 0.f;
              const float hxz = (a && c) ? a * c * pw[0][a ? a - 1 : 0] * pw[1][b] * pw[2][c ? c - 1 : 0] : 0.f;
              const float hyz = (b && c) ? b * c * pw[0][a] * pw[1][b ? b - 1 : 0] * pw[2][c ? c - 1 : 0] : 0.f;
              dn[0] = fmaf(s, hxx * h3[0] + hxy * h3[1] + hxz * h3[2], dn[0]);
              dn[1] = fmaf(s, hxy * h3[0] + hyy * h3[1] + hyz * h3[2], dn[1]);
              dn[2] = fmaf(s, hxz * h3[0] + hyz * h3[1] + hzz * h3[2], dn[2]);
            }
          }
        }
      }
      if (mode != 1) {
#pragma unroll
        for (int m = 0; m < 2 * LMAX + 1; ++m)
          if (m < m_count) out0[e * W + l * l + m] = y[m];
      }
      toff += d * m_count;
    }
    if (mode == 1) {
#pragma unroll
      for (int c = 0; c < 3; ++c) out0[3 * e + c] = dn[c];
    } else if (mode == 2) {
#pragma unroll
      for (int c = 0; c < 3; ++c) out1[3 * e + c] = dn[c];
    }
  }
}

using HarmFn = void (*)(const float*, const float*, const float*, const float*, float*, float*, int64_t, int);

static HarmFn harmonics_fn(int lmax) {
  switch (lmax) {
    case 1: return harmonics_kernel<1>;
    case 2: return harmonics_kernel<2>;
    case 3: return harmonics_kernel<3>;
    case 4: return harmonics_kernel<4>;
    case 5: return harmonics_kernel<5>;
    case 6: return harmonics_kernel<6>;
    default: return nullptr;
  }
}

}  // namespace ictc

using namespace ictc;

extern "C" int ictc_harmonics_table_size(int lmax) {
  int total = 0;
  for (int l = 1; l <= lmax; ++l) total += (l + 1) * (l + 2) / 2 * (2 * l + 1);
  return total;
}

extern "C" int ictc_direction_harmonics(const float* directions, const float* table, const float* grad_y,
                                        const float* grad_dir, float* out0, float* out1, int64_t rows, int lmax,
                                        int mode, void* stream) {
  if (rows < 0 || mode < 0 || mode > 2 || lmax < 1 || (rows > 0 && (!directions || !table || !out0)) ||
      (mode >= 1 && rows > 0 && !grad_y) || (mode == 2 && rows > 0 && (!grad_dir || !out1))) {
    ictc_set_error("ictc_direction_harmonics: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  HarmFn fn = harmonics_fn(lmax);
  if (!fn) {
    ictc_set_error("ictc_direction_harmonics: lmax must be in 1..6%s", "");
    return ICTC_ERR_UNSUPPORTED;
  }
  if (rows == 0) return ICTC_OK;
  int device = 0, sms = 0;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  int64_t blocks = (rows + kHarmThreads - 1) / kHarmThreads;
  int64_t cap = (int64_t)sms * 8;
  fn<<<(int)(blocks < cap ? blocks : cap), kHarmThreads, 0, (cudaStream_t)stream>>>(
      directions, table, grad_y, grad_dir, out0, out1, rows, mode);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error("direction harmonics launch failed: %s", cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}
