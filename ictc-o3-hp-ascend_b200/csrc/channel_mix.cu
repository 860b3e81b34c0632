// Equivariant channel mixing of one degree block in the flat [channel][2l+1] layout.
//
//   y[n, yoff + o*M + k] (+)= scale * sum_i W_s[o, i] * x[n, xoff + i*M + k]
//
// for every node n, with M = 2l+1 and W_s the weights of the node's species
// (S = 1 for species-independent linears).  This is the per-degree linear of the
// reference model: linear_up / product linear (EquivariantChannelLinearSO3,
// mace_ictc/models/pure_cartesian_ictd_fix.py:335-392), message_linear
// (PathPreservingLinearSO3, :629-661) and the element-conditioned self-connection
// (:2381-2440).  It reads and writes the flat feature rows in place, so a linear
// needs no degree-block slicing, concatenation or layout copies.
//
// One CTA: a tile of 32 nodes (contiguous, or a species-homogeneous node list) x
// 64 output channels.  Lane = node, warp = 8 consecutive output channels: per input
// channel a thread reads its node's M values (padded rows, no bank conflicts) and
// the warp's 8 weights as two broadcast float4 loads, for 8*M FMAs.  The reduction
// over input channels runs in chunks of 32 staged in shared memory.
#include <cstdint>
#include <cstdio>

#include "ictc_common.cuh"
#include "ictc_cuda.h"

void ictc_set_error(const char* fmt, const char* detail);

namespace ictc {
namespace {

constexpr int kOutTile = 64;      // output channels per CTA
constexpr int kOutPerWarp = 8;    // output channels per thread (8 warps)
constexpr int kTileNodes = 32;    // nodes per CTA (lane = node)
constexpr int kChunk = 32;        // input channels per shared-memory stage
constexpr int kWStride = kOutTile + 4;  // padded row of the transposed weight chunk

struct MixArgs {
  const float* x;
  const float* w;                 // [S, cout, cin]
  const int64_t* tiles;           // [T, kTileNodes] node ids (-1 padded) or null (contiguous tiles)
  const int32_t* tile_species;    // [T] or null
  float* y;
  int64_t x_stride, x_offset, y_stride, y_offset, nodes, num_tiles;
  int cin, cout;
  float scale;
  int accumulate;
};

template <int M>
__global__ void __launch_bounds__(256, (M <= 5) ? 2 : 1) channel_mix_kernel(MixArgs a) {
  extern __shared__ __align__(16) float smem[];
  constexpr int kXStride = kChunk * M + 1;        // odd: the 32 node rows hit distinct banks
  float* s_w = smem;                               // [kChunk][kWStride]: s_w[i][o] = W[o0 + o, i0 + i]
  float* s_x = smem + kChunk * kWStride;           // [kTileNodes][kXStride]
  __shared__ int64_t s_node[kTileNodes];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int o0 = blockIdx.y * kOutTile;
  const int ow = warp * kOutPerWarp;               // this warp's first output channel in the tile

  for (int64_t t = blockIdx.x; t < a.num_tiles; t += gridDim.x) {
    if (tid < kTileNodes) {
      int64_t n = -1;
      if (a.tiles) {
        n = a.tiles[t * kTileNodes + tid];
      } else {
        const int64_t c = t * kTileNodes + tid;
        n = c < a.nodes ? c : -1;
      }
      s_node[tid] = n;
    }
    __syncthreads();
    const int64_t node = s_node[lane];
    const int species = a.tile_species ? a.tile_species[t] : 0;
    const float* w = a.w + (int64_t)species * a.cout * a.cin;

    float acc[kOutPerWarp][M];
#pragma unroll
    for (int j = 0; j < kOutPerWarp; ++j)
#pragma unroll
      for (int k = 0; k < M; ++k) acc[j][k] = 0.f;

    // Register-staged pipeline: the loads of chunk c+1 are in flight while chunk c
    // is computed from shared memory.
    constexpr int kWPer = kChunk * kOutTile / 256;               // weight values per thread
    constexpr int kXPer = kTileNodes * kChunk * M / 256;         // input values per thread
    float rw[kWPer], rx[kXPer];
    auto fetch = [&](int i0) {
      const int kc = min(kChunk, a.cin - i0);
#pragma unroll
      for (int q = 0; q < kWPer; ++q) {
        const int idx = tid + 256 * q, i = idx % kChunk, ol = idx / kChunk;
        rw[q] = (i < kc && o0 + ol < a.cout) ? __ldg(w + (int64_t)(o0 + ol) * a.cin + i0 + i) : 0.f;
      }
#pragma unroll
      for (int q = 0; q < kXPer; ++q) {
        const int idx = tid + 256 * q, nl = idx / (kChunk * M), r = idx % (kChunk * M);
        const int64_t n = s_node[nl];
        rx[q] = (n >= 0 && r < kc * M) ? __ldg(a.x + n * a.x_stride + a.x_offset + (int64_t)i0 * M + r) : 0.f;
      }
    };
    fetch(0);
    for (int i0 = 0; i0 < a.cin; i0 += kChunk) {
      const int kc = min(kChunk, a.cin - i0);
#pragma unroll
      for (int q = 0; q < kWPer; ++q) {
        const int idx = tid + 256 * q, i = idx % kChunk, ol = idx / kChunk;
        s_w[i * kWStride + ol] = rw[q];
      }
#pragma unroll
      for (int q = 0; q < kXPer; ++q) {
        const int idx = tid + 256 * q, nl = idx / (kChunk * M), r = idx % (kChunk * M);
        s_x[nl * kXStride + r] = rx[q];
      }
      __syncthreads();
      if (i0 + kChunk < a.cin) fetch(i0 + kChunk);
      const float* xr = s_x + lane * kXStride;
#pragma unroll 4
      for (int i = 0; i < kc; ++i) {
        const float4 w0 = *reinterpret_cast<const float4*>(s_w + i * kWStride + ow);
        const float4 w1 = *reinterpret_cast<const float4*>(s_w + i * kWStride + ow + 4);
        const float wv[kOutPerWarp] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float xv[M];
#pragma unroll
        for (int k = 0; k < M; ++k) xv[k] = xr[i * M + k];
#pragma unroll
        for (int j = 0; j < kOutPerWarp; ++j)
#pragma unroll
          for (int k = 0; k < M; ++k) acc[j][k] = fmaf(wv[j], xv[k], acc[j][k]);
      }
      __syncthreads();
    }
    if (node >= 0) {
      float* yr = a.y + node * a.y_stride + a.y_offset;
#pragma unroll
      for (int j = 0; j < kOutPerWarp; ++j) {
        const int o = o0 + ow + j;
        if (o >= a.cout) break;
#pragma unroll
        for (int k = 0; k < M; ++k)
          yr[o * M + k] = a.accumulate ? yr[o * M + k] + a.scale * acc[j][k] : a.scale * acc[j][k];
      }
    }
  }
}

template <int M>
int launch(const MixArgs& a, cudaStream_t stream) {
  const size_t smem = sizeof(float) * (kChunk * kWStride + kTileNodes * (kChunk * M + 1));
  static_assert(sizeof(float) * (kChunk * kWStride + kTileNodes * (kChunk * 7 + 1)) <= 48 * 1024,
                "fits the default dynamic shared memory");
  int device = 0, sms = 0;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int ytiles = (a.cout + kOutTile - 1) / kOutTile;
  int64_t grid = a.num_tiles;
  const int64_t cap = (int64_t)sms * 8 / ytiles + 1;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  channel_mix_kernel<M><<<dim3((unsigned)grid, (unsigned)ytiles), 256, smem, stream>>>(a);
  return ICTC_OK;
}

}  // namespace
}  // namespace ictc

using namespace ictc;

extern "C" int ictc_channel_mix_tile_nodes(void) { return kTileNodes; }

extern "C" int ictc_channel_mix(const float* x, int64_t x_stride, int64_t x_offset, const float* weight,
                                const int64_t* tiles, const int32_t* tile_species, int64_t num_tiles, float* y,
                                int64_t y_stride, int64_t y_offset, int64_t nodes, int cin, int cout, int degree,
                                float scale, int accumulate, void* stream) {
  if (nodes < 0 || cin < 1 || cout < 1 || degree < 0 || degree > 3 || !weight || (nodes > 0 && (!x || !y)) ||
      (tiles && num_tiles < 0) || (tiles == nullptr && tile_species != nullptr)) {
    ictc_set_error("ictc_channel_mix: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  if (nodes == 0) return ICTC_OK;
  MixArgs a;
  a.x = x;
  a.w = weight;
  a.tiles = tiles;
  a.tile_species = tile_species;
  a.y = y;
  a.x_stride = x_stride;
  a.x_offset = x_offset;
  a.y_stride = y_stride;
  a.y_offset = y_offset;
  a.nodes = nodes;
  a.num_tiles = tiles ? num_tiles : (nodes + kTileNodes - 1) / kTileNodes;
  a.cin = cin;
  a.cout = cout;
  a.scale = scale;
  a.accumulate = accumulate;
  if (a.num_tiles == 0) return ICTC_OK;
  cudaStream_t s = (cudaStream_t)stream;
  switch (degree) {
    case 0: launch<1>(a, s); break;
    case 1: launch<3>(a, s); break;
    case 2: launch<5>(a, s); break;
    default: launch<7>(a, s); break;
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error("ictc_channel_mix: %s", cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}
