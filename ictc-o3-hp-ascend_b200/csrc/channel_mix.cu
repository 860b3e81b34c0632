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
// One CTA: a tile of kTileNodes nodes (contiguous, or species-homogeneous node
// lists) x 64 output channels.  The reduction over input channels runs in chunks
// of kChunk: the chunk of W (transposed into shared memory) and the tile's input
// rows are staged in shared memory; thread (o, g) accumulates its output channel o
// for the nodes g, g+4, g+8, g+12 of the tile.
#include <cstdint>
#include <cstdio>

#include "ictc_common.cuh"
#include "ictc_cuda.h"

void ictc_set_error(const char* fmt, const char* detail);

namespace ictc {
namespace {

constexpr int kOutTile = 64;      // output channels per CTA
constexpr int kGroups = 4;        // node groups per CTA (256 threads)
constexpr int kNodesPerThread = 4;
constexpr int kTileNodes = kGroups * kNodesPerThread;  // 16
constexpr int kChunk = 64;        // input channels per shared-memory stage

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
__global__ void __launch_bounds__(256) channel_mix_kernel(MixArgs a) {
  extern __shared__ __align__(16) float smem[];
  float* s_w = smem;                               // [kChunk][kOutTile + 1] (padded: no bank conflicts)
  float* s_x = smem + kChunk * (kOutTile + 1);     // [kTileNodes][kChunk * M]
  const int tid = threadIdx.x;
  const int o_local = tid % kOutTile, g = tid / kOutTile;
  const int o0 = blockIdx.y * kOutTile;
  const int o = o0 + o_local;

  for (int64_t t = blockIdx.x; t < a.num_tiles; t += gridDim.x) {
    int64_t node[kNodesPerThread];
    __shared__ int64_t s_node[kTileNodes];
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
#pragma unroll
    for (int j = 0; j < kNodesPerThread; ++j) node[j] = s_node[g + kGroups * j];
    const int species = a.tile_species ? a.tile_species[t] : 0;
    const float* w = a.w + (int64_t)species * a.cout * a.cin;

    float acc[kNodesPerThread][M];
#pragma unroll
    for (int j = 0; j < kNodesPerThread; ++j)
#pragma unroll
      for (int k = 0; k < M; ++k) acc[j][k] = 0.f;

    for (int i0 = 0; i0 < a.cin; i0 += kChunk) {
      const int kc = min(kChunk, a.cin - i0);
      // W chunk, transposed: s_w[i][o_local] = W[o0 + o_local, i0 + i].
      for (int idx = tid; idx < kChunk * kOutTile; idx += blockDim.x) {
        const int i = idx % kChunk, ol = idx / kChunk;
        s_w[i * (kOutTile + 1) + ol] = (i < kc && o0 + ol < a.cout) ? __ldg(w + (int64_t)(o0 + ol) * a.cin + i0 + i) : 0.f;
      }
      // Input rows of the tile: kc * M contiguous floats per node.
      for (int idx = tid; idx < kTileNodes * kChunk * M; idx += blockDim.x) {
        const int nl = idx / (kChunk * M), r = idx % (kChunk * M);
        const int64_t n = s_node[nl];
        s_x[idx] = (n >= 0 && r < kc * M) ? __ldg(a.x + n * a.x_stride + a.x_offset + (int64_t)i0 * M + r) : 0.f;
      }
      __syncthreads();
#pragma unroll 4
      for (int i = 0; i < kc; ++i) {
        const float wv = s_w[i * (kOutTile + 1) + o_local];
#pragma unroll
        for (int j = 0; j < kNodesPerThread; ++j) {
          const float* xr = s_x + (g + kGroups * j) * (kChunk * M) + i * M;
#pragma unroll
          for (int k = 0; k < M; ++k) acc[j][k] = fmaf(wv, xr[k], acc[j][k]);
        }
      }
      __syncthreads();
    }
    if (o < a.cout) {
#pragma unroll
      for (int j = 0; j < kNodesPerThread; ++j) {
        if (node[j] < 0) continue;
        float* yr = a.y + node[j] * a.y_stride + a.y_offset + (int64_t)o * M;
#pragma unroll
        for (int k = 0; k < M; ++k) yr[k] = a.accumulate ? yr[k] + a.scale * acc[j][k] : a.scale * acc[j][k];
      }
    }
  }
}

template <int M>
int launch(const MixArgs& a, cudaStream_t stream) {
  const size_t smem = sizeof(float) * (kChunk * (kOutTile + 1) + kTileNodes * kChunk * M);
  static_assert(sizeof(float) * (kChunk * (kOutTile + 1) + kTileNodes * kChunk * 7) <= 48 * 1024,
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
