// Edge geometry of the MACE-ICTC interaction: for an edge vector v,
//   r = |v|,  unit = v / max(r, 1e-8),  mask = (r <= r_max),
//   radial[b] = sqrt(2 / r_max) sin(w_b r) / max(r, 1e-12) * env(r) * (sqrt(B) if normed),
//   w_b = (pi / r_max) (b + 1),  b = 0 .. B-1,
//   env(r) = 1 - (p+1)(p+2)/2 x^p + p(p+2) x^(p+1) - p(p+1)/2 x^(p+2),  x = r / r_max,  0 for r >= r_max
// (Bessel basis and polynomial envelope of mace_ictc/models/radial_basis.py:42-91
// and :11-39; unit directions as in the model's edge_features), and the adjoint
// dL/dv from dL/dunit and dL/dradial.  One thread per edge: the whole chain of
// elementwise ops and the reduction over the basis stay in registers (one read of
// v, one write per output).
#include "ictc_common.cuh"
#include "ictc_cuda.h"

#include <cmath>
#include <cstdio>

void ictc_set_error(const char* fmt, const char* detail);

namespace ictc {
namespace {

constexpr int kGeoThreads = 256;
constexpr int kMaxBasis = 16;

struct GeoArgs {
  const float* vec;
  const float* grad_unit;     // backward: [E, 3] or null
  const float* grad_radial;   // backward: [E, B] or null
  float* unit;                // forward outputs
  float* radial;
  float* mask;
  float* grad_vec;            // backward output
  int64_t edges;
  float r_max, inv_r_max, freq, prefactor;
  int basis, p;
};

__device__ __forceinline__ float ipow(float x, int n) {
  float y = 1.f;
  for (int i = 0; i < n; ++i) y *= x;
  return y;
}

// Envelope and its derivative with respect to r.
__device__ __forceinline__ void envelope(const GeoArgs& a, float r, float& env, float& denv) {
  const float x = r * a.inv_r_max;
  const float pf = (float)a.p;
  const float c0 = (pf + 1.f) * (pf + 2.f) / 2.f, c1 = pf * (pf + 2.f), c2 = pf * (pf + 1.f) / 2.f;
  const float xp1 = a.p >= 1 ? ipow(x, a.p - 1) : 0.f;   // x^(p-1)
  const float xp = xp1 * x, xq = xp * x, xr = xq * x;   // x^p, x^(p+1), x^(p+2)
  const bool within = r < a.r_max;
  env = within ? (1.f - c0 * xp + c1 * xq - c2 * xr) : 0.f;
  denv = within ? a.inv_r_max * (-c0 * pf * xp1 + c1 * (pf + 1.f) * xp - c2 * (pf + 2.f) * xq) : 0.f;
}

__global__ void __launch_bounds__(kGeoThreads) edge_geometry_kernel(GeoArgs a) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < a.edges;
       e += (int64_t)gridDim.x * blockDim.x) {
    const float vx = a.vec[3 * e], vy = a.vec[3 * e + 1], vz = a.vec[3 * e + 2];
    const float r = sqrtf(vx * vx + vy * vy + vz * vz);
    const float rn = fmaxf(r, 1e-8f);
    a.unit[3 * e] = vx / rn;
    a.unit[3 * e + 1] = vy / rn;
    a.unit[3 * e + 2] = vz / rn;
    a.mask[e] = r <= a.r_max ? 1.f : 0.f;
    float env, denv;
    envelope(a, r, env, denv);
    const float rb = fmaxf(r, 1e-12f);
    for (int b = 0; b < a.basis; ++b) {
      const float w = a.freq * (float)(b + 1);
      a.radial[e * a.basis + b] = a.prefactor * sinf(r * w) / rb * env;
    }
  }
}

__global__ void __launch_bounds__(kGeoThreads) edge_geometry_backward_kernel(GeoArgs a) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < a.edges;
       e += (int64_t)gridDim.x * blockDim.x) {
    const float vx = a.vec[3 * e], vy = a.vec[3 * e + 1], vz = a.vec[3 * e + 2];
    const float r = sqrtf(vx * vx + vy * vy + vz * vz);
    float gx = 0.f, gy = 0.f, gz = 0.f;
    // Through the unit vector: (g - u (u . g)) / r, or g / 1e-8 where the floor applies.
    if (a.grad_unit) {
      const float ux = a.grad_unit[3 * e], uy = a.grad_unit[3 * e + 1], uz = a.grad_unit[3 * e + 2];
      if (r > 1e-8f) {
        const float inv = 1.f / r;
        const float nx = vx * inv, ny = vy * inv, nz = vz * inv;
        const float d = nx * ux + ny * uy + nz * uz;
        gx = (ux - nx * d) * inv;
        gy = (uy - ny * d) * inv;
        gz = (uz - nz * d) * inv;
      } else {
        gx = ux * 1e8f;
        gy = uy * 1e8f;
        gz = uz * 1e8f;
      }
    }
    // Through the radial embedding: dL/dr = sum_b g_b d radial_b / dr, then dr/dv = v / r.
    if (a.grad_radial && r > 1e-12f) {
      float env, denv;
      envelope(a, r, env, denv);
      const float inv_r = 1.f / r;
      float gr = 0.f;
      for (int b = 0; b < a.basis; ++b) {
        const float w = a.freq * (float)(b + 1);
        const float t = r * w;
        float s, c;
        sincosf(t, &s, &c);
        // d/dr [sin(w r) / r] = (t cos t - sin t) / r^2: the two terms cancel for small
        // t, so there the series w^2 (-t/3 + t^3/30 - t^5/840) is used.
        float fprime;
        if (t < 0.5f) {
          const float t2 = t * t;
          fprime = w * w * t * (-1.f / 3.f + t2 * (1.f / 30.f - t2 * (1.f / 840.f)));
        } else {
          fprime = (t * c - s) * inv_r * inv_r;
        }
        const float df = a.prefactor * (fprime * env + s * inv_r * denv);
        gr = fmaf(a.grad_radial[e * a.basis + b], df, gr);
      }
      gx = fmaf(gr, vx * inv_r, gx);
      gy = fmaf(gr, vy * inv_r, gy);
      gz = fmaf(gr, vz * inv_r, gz);
    }
    a.grad_vec[3 * e] = gx;
    a.grad_vec[3 * e + 1] = gy;
    a.grad_vec[3 * e + 2] = gz;
  }
}

GeoArgs make_args(const float* vec, int64_t edges, float r_max, int num_basis, int p, int basis_norm) {
  GeoArgs a{};
  a.vec = vec;
  a.edges = edges;
  a.r_max = r_max;
  a.inv_r_max = 1.f / r_max;
  a.freq = (float)(M_PI / (double)r_max);
  a.prefactor = (float)(std::sqrt(2.0 / (double)r_max) * (basis_norm ? std::sqrt((double)num_basis) : 1.0));
  a.basis = num_basis;
  a.p = p;
  return a;
}

int launch_geo(bool backward, const GeoArgs& a, void* stream, const char* what) {
  int device = 0, sms = 0;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  int64_t blocks = (a.edges + kGeoThreads - 1) / kGeoThreads;
  const int64_t cap = (int64_t)sms * 8;
  if (blocks > cap) blocks = cap;
  if (backward)
    edge_geometry_backward_kernel<<<(int)blocks, kGeoThreads, 0, (cudaStream_t)stream>>>(a);
  else
    edge_geometry_kernel<<<(int)blocks, kGeoThreads, 0, (cudaStream_t)stream>>>(a);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error(what, cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}

}  // namespace
}  // namespace ictc

using namespace ictc;

extern "C" int ictc_edge_geometry(const float* vec, int64_t edges, float r_max, int num_basis, int p,
                                  int basis_norm, float* unit, float* radial, float* mask, void* stream) {
  if (edges < 0 || !(r_max > 0.f) || num_basis < 1 || num_basis > kMaxBasis || p < 1 ||
      (edges > 0 && (!vec || !unit || !radial || !mask))) {
    ictc_set_error("ictc_edge_geometry: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  if (edges == 0) return ICTC_OK;
  GeoArgs a = make_args(vec, edges, r_max, num_basis, p, basis_norm);
  a.unit = unit;
  a.radial = radial;
  a.mask = mask;
  return launch_geo(false, a, stream, "edge geometry launch failed: %s");
}

extern "C" int ictc_edge_geometry_backward(const float* vec, const float* grad_unit, const float* grad_radial,
                                           int64_t edges, float r_max, int num_basis, int p, int basis_norm,
                                           float* grad_vec, void* stream) {
  if (edges < 0 || !(r_max > 0.f) || num_basis < 1 || num_basis > kMaxBasis || p < 1 ||
      (edges > 0 && (!vec || !grad_vec))) {
    ictc_set_error("ictc_edge_geometry_backward: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  if (edges == 0) return ICTC_OK;
  GeoArgs a = make_args(vec, edges, r_max, num_basis, p, basis_norm);
  a.grad_unit = grad_unit;
  a.grad_radial = grad_radial;
  a.grad_vec = grad_vec;
  return launch_geo(true, a, stream, "edge geometry backward launch failed: %s");
}
