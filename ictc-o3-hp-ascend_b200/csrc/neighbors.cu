// Periodic cell-list neighbour search on sm_100a.
//
// Replaces the reference's torch-only PBC radius graph
// (mace_ictc/utils/graph_utils.py:217-297, which needs torch_cluster) for an
// orthorhombic periodic box with cutoff < half of every box length and at least
// three cells per axis.  Output is the destination-sorted edge list the message
// kernels consume: for receiver i (dst), its neighbours j (src) with
//   pos[i] - pos[j] + shift = minimum-image vector,  |.| < cutoff,
// grouped by i (offsets[i] .. offsets[i+1]), and inside a receiver ordered by
// the 27 neighbour cells (z, y, x offsets -1..1) then by atom id, so the list is
// deterministic.
//
// Phases (all on the caller's stream):
//   1 bin:    cell of every atom, per-cell counts (atomics on counts only)
//   2 scan:   cell starts
//   3 place:  atoms into their cell's range; each cell's range sorted by id
//   4 count:  neighbours per atom, exclusive scan -> offsets (dst CSR)
//   5 fill:   src, dst, shift per edge
// Phases 1-4 are ictc_neighbor_count, phase 5 is ictc_neighbor_fill; the
// workspace carries the cell lists from one to the other.
#include "ictc_common.cuh"
#include "ictc_cuda.h"

#include <cmath>
#include <cstdio>

void ictc_set_error(const char* fmt, const char* detail);

namespace ictc {

struct CellGrid {
  int nx, ny, nz;
  float lx, ly, lz;
  float cutoff2;
  int64_t cells() const { return (int64_t)nx * ny * nz; }
};

struct NeighborWorkspace {
  int32_t* cell_of_atom;  // [N]
  int32_t* cell_count;    // [cells]
  int32_t* cell_start;    // [cells + 1]
  int32_t* cell_fill;     // [cells]
  int32_t* sorted_atoms;  // [N]
  int32_t* atom_count;    // [N] neighbours per atom
};

__host__ __device__ inline size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

static size_t workspace_layout(int64_t atoms, int64_t cells, NeighborWorkspace* ws, char* base) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> char* {
    char* p = base ? base + off : nullptr;
    off += align256(bytes);
    return p;
  };
  char* a = take(sizeof(int32_t) * atoms);
  char* b = take(sizeof(int32_t) * cells);
  char* c = take(sizeof(int32_t) * (cells + 1));
  char* d = take(sizeof(int32_t) * cells);
  char* e = take(sizeof(int32_t) * atoms);
  char* f = take(sizeof(int32_t) * atoms);
  if (ws) {
    ws->cell_of_atom = (int32_t*)a; ws->cell_count = (int32_t*)b; ws->cell_start = (int32_t*)c;
    ws->cell_fill = (int32_t*)d; ws->sorted_atoms = (int32_t*)e; ws->atom_count = (int32_t*)f;
  }
  return off;
}

static bool make_grid(const float* box, float cutoff, CellGrid* g) {
  if (!(cutoff > 0.f) || !(box[0] > 0.f) || !(box[1] > 0.f) || !(box[2] > 0.f)) return false;
  if (2.f * cutoff >= box[0] || 2.f * cutoff >= box[1] || 2.f * cutoff >= box[2]) return false;
  g->nx = (int)floorf(box[0] / cutoff);
  g->ny = (int)floorf(box[1] / cutoff);
  g->nz = (int)floorf(box[2] / cutoff);
  if (g->nx < 3 || g->ny < 3 || g->nz < 3) return false;
  g->lx = box[0]; g->ly = box[1]; g->lz = box[2];
  g->cutoff2 = cutoff * cutoff;
  return true;
}

__device__ __forceinline__ float wrap(float p, float l) { return p - l * floorf(p / l); }

__device__ __forceinline__ int cell_coord(float p, float l, int n) {
  int c = (int)(wrap(p, l) / l * n);
  return c < 0 ? 0 : (c >= n ? n - 1 : c);
}

__global__ void bin_kernel(const float* __restrict__ pos, int64_t atoms, CellGrid g, NeighborWorkspace ws) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < atoms; i += (int64_t)gridDim.x * blockDim.x) {
    const int cx = cell_coord(pos[3 * i], g.lx, g.nx);
    const int cy = cell_coord(pos[3 * i + 1], g.ly, g.ny);
    const int cz = cell_coord(pos[3 * i + 2], g.lz, g.nz);
    const int cell = (cz * g.ny + cy) * g.nx + cx;
    ws.cell_of_atom[i] = cell;
    atomicAdd(ws.cell_count + cell, 1);
  }
}

// Exclusive scan of `n` int32 (or int64 output) values in one CTA, tile by tile.
template <class In, class Out>
__global__ void scan_kernel(const In* __restrict__ in, Out* __restrict__ out, int64_t n) {
  __shared__ Out s_tile[1024];
  __shared__ Out s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < n; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    Out v = i < n ? (Out)in[i] : (Out)0;
    s_tile[threadIdx.x] = v;
    __syncthreads();
    for (int o = 1; o < (int)blockDim.x; o <<= 1) {
      Out add = threadIdx.x >= (unsigned)o ? s_tile[threadIdx.x - o] : (Out)0;
      __syncthreads();
      s_tile[threadIdx.x] += add;
      __syncthreads();
    }
    if (i < n) out[i] = s_carry + s_tile[threadIdx.x] - v;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) s_carry += s_tile[threadIdx.x];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[n] = s_carry;
}

__global__ void place_kernel(int64_t atoms, NeighborWorkspace ws) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < atoms; i += (int64_t)gridDim.x * blockDim.x) {
    const int cell = ws.cell_of_atom[i];
    const int slot = atomicAdd(ws.cell_fill + cell, 1);
    ws.sorted_atoms[ws.cell_start[cell] + slot] = (int32_t)i;
  }
}

// Insertion sort of each cell's atom ids (cells hold a handful of atoms).
__global__ void sort_cells_kernel(int64_t cells, NeighborWorkspace ws) {
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < cells; c += (int64_t)gridDim.x * blockDim.x) {
    int32_t* a = ws.sorted_atoms + ws.cell_start[c];
    const int n = ws.cell_start[c + 1] - ws.cell_start[c];
    for (int k = 1; k < n; ++k) {
      const int32_t v = a[k];
      int j = k - 1;
      while (j >= 0 && a[j] > v) {
        a[j + 1] = a[j];
        --j;
      }
      a[j + 1] = v;
    }
  }
}

// Count (FILL = false) or write (FILL = true) the neighbours of the receivers
// (atoms [0, receivers)); sources range over all binned atoms.
template <bool FILL>
__global__ void neighbor_kernel(const float* __restrict__ pos, int64_t receivers, CellGrid g, NeighborWorkspace ws,
                                int32_t* __restrict__ counts, const int64_t* __restrict__ offsets,
                                int64_t* __restrict__ src, int64_t* __restrict__ dst, float* __restrict__ shift) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < receivers;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float px = pos[3 * i], py = pos[3 * i + 1], pz = pos[3 * i + 2];
    const int cell = ws.cell_of_atom[i];
    const int cx = cell % g.nx, cy = (cell / g.nx) % g.ny, cz = cell / (g.nx * g.ny);
    int found = 0;
    int64_t out = FILL ? offsets[i] : 0;
    for (int dz = -1; dz <= 1; ++dz) {
      const int z = (cz + dz + g.nz) % g.nz;
      for (int dy = -1; dy <= 1; ++dy) {
        const int y = (cy + dy + g.ny) % g.ny;
        for (int dx = -1; dx <= 1; ++dx) {
          const int x = (cx + dx + g.nx) % g.nx;
          const int c = (z * g.ny + y) * g.nx + x;
          for (int k = ws.cell_start[c]; k < ws.cell_start[c + 1]; ++k) {
            const int32_t j = ws.sorted_atoms[k];
            if (j == i) continue;
            // Minimum-image vector pos[i] - pos[j] + shift.
            const float rx = px - pos[3 * j], ry = py - pos[3 * j + 1], rz = pz - pos[3 * j + 2];
            const float sx = -g.lx * rintf(rx / g.lx), sy = -g.ly * rintf(ry / g.ly), sz = -g.lz * rintf(rz / g.lz);
            const float vx = rx + sx, vy = ry + sy, vz = rz + sz;
            if (vx * vx + vy * vy + vz * vz < g.cutoff2) {
              if (FILL) {
                src[out] = j;
                dst[out] = i;
                shift[3 * out] = sx;
                shift[3 * out + 1] = sy;
                shift[3 * out + 2] = sz;
                ++out;
              } else {
                ++found;
              }
            }
          }
        }
      }
    }
    if (!FILL) counts[i] = found;
  }
}

static int grid_size(int64_t n, int threads) {
  int device = 0, sms = 0;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  int64_t blocks = (n + threads - 1) / threads;
  int64_t cap = (int64_t)sms * 8;
  if (blocks < 1) blocks = 1;
  return (int)(blocks < cap ? blocks : cap);
}

}  // namespace ictc

using namespace ictc;

extern "C" int64_t ictc_neighbor_workspace_bytes(int64_t atoms, const float* box, float cutoff) {
  CellGrid g;
  if (!box || atoms < 0 || !make_grid(box, cutoff, &g)) return -1;
  return (int64_t)workspace_layout(atoms, g.cells(), nullptr, nullptr);
}

static int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error(what, cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}

static int prepare(const float* pos, int64_t atoms, const float* box, float cutoff, const void* workspace,
                   int64_t workspace_bytes, const int64_t* offsets, CellGrid* g, NeighborWorkspace* ws,
                   const char* who) {
  if (!box || !make_grid(box, cutoff, g)) {
    ictc_set_error("%s: unsupported box (need cutoff < L/2 and >= 3 cells per axis)", who);
    return ICTC_ERR_UNSUPPORTED;
  }
  if (atoms < 0 || atoms > INT32_MAX || !offsets || (atoms > 0 && (!pos || !workspace))) {
    ictc_set_error("%s: invalid argument", who);
    return ICTC_ERR_INVALID;
  }
  size_t need = workspace_layout(atoms, g->cells(), ws, (char*)workspace);
  if (workspace_bytes < 0 || (size_t)workspace_bytes < need) {
    ictc_set_error("%s: workspace too small", who);
    return ICTC_ERR_INVALID;
  }
  return ICTC_OK;
}

static int neighbor_count(const float* pos, int64_t atoms, int64_t receivers, const float* box, float cutoff,
                          void* workspace, int64_t workspace_bytes, int64_t* offsets, void* stream, const char* who) {
  CellGrid g;
  NeighborWorkspace ws;
  int status = prepare(pos, atoms, box, cutoff, workspace, workspace_bytes, offsets, &g, &ws, who);
  if (status != ICTC_OK) return status;
  if (receivers < 0 || receivers > atoms) {
    ictc_set_error("%s: receivers must lie in [0, atoms]", who);
    return ICTC_ERR_INVALID;
  }
  cudaStream_t s = (cudaStream_t)stream;
  if (receivers == 0) {
    cudaMemsetAsync(offsets, 0, sizeof(int64_t), s);
    return check_launch("neighbour count: %s");
  }
  const int64_t cells = g.cells();
  cudaMemsetAsync(ws.cell_count, 0, sizeof(int32_t) * cells, s);
  cudaMemsetAsync(ws.cell_fill, 0, sizeof(int32_t) * cells, s);
  bin_kernel<<<grid_size(atoms, 256), 256, 0, s>>>(pos, atoms, g, ws);
  scan_kernel<int32_t, int32_t><<<1, 1024, 0, s>>>(ws.cell_count, ws.cell_start, cells);
  place_kernel<<<grid_size(atoms, 256), 256, 0, s>>>(atoms, ws);
  sort_cells_kernel<<<grid_size(cells, 128), 128, 0, s>>>(cells, ws);
  neighbor_kernel<false><<<grid_size(receivers, 128), 128, 0, s>>>(pos, receivers, g, ws, ws.atom_count, nullptr,
                                                                    nullptr, nullptr, nullptr);
  scan_kernel<int32_t, int64_t><<<1, 1024, 0, s>>>(ws.atom_count, offsets, receivers);
  return check_launch("neighbour count: %s");
}

static int neighbor_fill(const float* pos, int64_t atoms, int64_t receivers, const float* box, float cutoff,
                         const void* workspace, int64_t workspace_bytes, const int64_t* offsets, int64_t* src,
                         int64_t* dst, float* shift, void* stream, const char* who) {
  CellGrid g;
  NeighborWorkspace ws;
  int status = prepare(pos, atoms, box, cutoff, workspace, workspace_bytes, offsets, &g, &ws, who);
  if (status != ICTC_OK) return status;
  if (receivers < 0 || receivers > atoms) {
    ictc_set_error("%s: receivers must lie in [0, atoms]", who);
    return ICTC_ERR_INVALID;
  }
  if (receivers == 0) return ICTC_OK;
  if (!src || !dst || !shift) {
    ictc_set_error("%s: invalid argument", who);
    return ICTC_ERR_INVALID;
  }
  neighbor_kernel<true><<<grid_size(receivers, 128), 128, 0, (cudaStream_t)stream>>>(pos, receivers, g, ws, nullptr,
                                                                                       offsets, src, dst, shift);
  return check_launch("neighbour fill: %s");
}

extern "C" int ictc_neighbor_count(const float* pos, int64_t atoms, const float* box, float cutoff, void* workspace,
                                   int64_t workspace_bytes, int64_t* offsets, void* stream) {
  return neighbor_count(pos, atoms, atoms, box, cutoff, workspace, workspace_bytes, offsets, stream,
                        "ictc_neighbor_count");
}

extern "C" int ictc_neighbor_fill(const float* pos, int64_t atoms, const float* box, float cutoff,
                                  const void* workspace, int64_t workspace_bytes, const int64_t* offsets,
                                  int64_t* src, int64_t* dst, float* shift, void* stream) {
  return neighbor_fill(pos, atoms, atoms, box, cutoff, workspace, workspace_bytes, offsets, src, dst, shift, stream,
                       "ictc_neighbor_fill");
}

extern "C" int ictc_neighbor_count_receivers(const float* pos, int64_t atoms, int64_t receivers, const float* box,
                                             float cutoff, void* workspace, int64_t workspace_bytes,
                                             int64_t* offsets, void* stream) {
  return neighbor_count(pos, atoms, receivers, box, cutoff, workspace, workspace_bytes, offsets, stream,
                        "ictc_neighbor_count_receivers");
}

extern "C" int ictc_neighbor_fill_receivers(const float* pos, int64_t atoms, int64_t receivers, const float* box,
                                            float cutoff, const void* workspace, int64_t workspace_bytes,
                                            const int64_t* offsets, int64_t* src, int64_t* dst, float* shift,
                                            void* stream) {
  return neighbor_fill(pos, atoms, receivers, box, cutoff, workspace, workspace_bytes, offsets, src, dst, shift,
                       stream, "ictc_neighbor_fill_receivers");
}

// ---------------------------------------------------------------------------
// Allocation-free variant (no counterpart in the reference).
//
// Some callers cannot allocate device memory while they run a step: an MD
// engine that owns every device buffer through its own pool, a host program
// linking this C library without a CUDA-aware allocator to hand out scratch, or
// code that must not call cudaMalloc inside a time-critical loop.  For them the
// search below keeps its scratch (the cell lists) in a file-scope device array
// of fixed size, so the caller only provides the outputs.
// ---------------------------------------------------------------------------

#include <mutex>

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB, held by every GPU that loads the library
static __device__ __align__(256) unsigned char g_neighbor_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
static std::mutex g_scratch_mutex;
static void* g_scratch_address[kMaxDevices] = {};

// Device address of g_neighbor_scratch on the current device (host code must not use
// the symbol's host-side name as a device pointer).  Looked up with the device current
// on every call that is not being captured into a CUDA graph, so a context that was
// torn down and re-created (cudaDeviceReset) never leaves a stale address behind;
// captured calls use the address of the last uncaptured call on that device, and a
// device's first call must therefore not be captured.
static int scratch_address(cudaStream_t stream, void** out) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
    cudaGetLastError();
    ictc_set_error("ictc_neighbor_list_noalloc: no usable current device%s", "");
    return ICTC_ERR_CUDA;
  }
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &capture) != cudaSuccess) {
    cudaGetLastError();
    capture = cudaStreamCaptureStatusActive;  // unknown: do not call into the runtime's module table
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (capture == cudaStreamCaptureStatusNone) {
    void* ptr = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&ptr, g_neighbor_scratch);
    if (err != cudaSuccess || !ptr) {
      cudaGetLastError();
      ictc_set_error("ictc_neighbor_list_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(err));
      return ICTC_ERR_CUDA;
    }
    g_scratch_address[device] = ptr;
  } else if (!g_scratch_address[device]) {
    ictc_set_error("ictc_neighbor_list_noalloc: the first call on a device must not be captured%s", "");
    return ICTC_ERR_INVALID;
  }
  *out = g_scratch_address[device];
  return ICTC_OK;
}

// Fill phase that writes only when the edge count fits the caller's capacity.
__global__ void neighbor_fill_capped_kernel(const float* __restrict__ pos, int64_t atoms, CellGrid g,
                                            NeighborWorkspace ws, const int64_t* __restrict__ offsets,
                                            int64_t max_edges, int64_t* __restrict__ src, int64_t* __restrict__ dst,
                                            float* __restrict__ shift) {
  if (offsets[atoms] > max_edges) return;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < atoms; i += (int64_t)gridDim.x * blockDim.x) {
    const float px = pos[3 * i], py = pos[3 * i + 1], pz = pos[3 * i + 2];
    const int cell = ws.cell_of_atom[i];
    const int cx = cell % g.nx, cy = (cell / g.nx) % g.ny, cz = cell / (g.nx * g.ny);
    int64_t out = offsets[i];
    for (int dz = -1; dz <= 1; ++dz) {
      const int z = (cz + dz + g.nz) % g.nz;
      for (int dy = -1; dy <= 1; ++dy) {
        const int y = (cy + dy + g.ny) % g.ny;
        for (int dx = -1; dx <= 1; ++dx) {
          const int x = (cx + dx + g.nx) % g.nx;
          const int c = (z * g.ny + y) * g.nx + x;
          for (int k = ws.cell_start[c]; k < ws.cell_start[c + 1]; ++k) {
            const int32_t j = ws.sorted_atoms[k];
            if (j == i) continue;
            const float rx = px - pos[3 * j], ry = py - pos[3 * j + 1], rz = pz - pos[3 * j + 2];
            const float sx = -g.lx * rintf(rx / g.lx), sy = -g.ly * rintf(ry / g.ly), sz = -g.lz * rintf(rz / g.lz);
            const float vx = rx + sx, vy = ry + sy, vz = rz + sz;
            if (vx * vx + vy * vy + vz * vz < g.cutoff2) {
              src[out] = j;
              dst[out] = i;
              shift[3 * out] = sx;
              shift[3 * out + 1] = sy;
              shift[3 * out + 2] = sz;
              ++out;
            }
          }
        }
      }
    }
  }
}

}  // namespace

extern "C" int64_t ictc_neighbor_noalloc_scratch_bytes(void) { return (int64_t)kNoAllocScratchBytes; }

extern "C" int ictc_neighbor_list_noalloc(const float* pos, int64_t atoms, const float* box, float cutoff,
                                          int64_t* offsets, int64_t* src, int64_t* dst, float* shift,
                                          int64_t max_edges, void* stream) {
  CellGrid g;
  if (!box || !make_grid(box, cutoff, &g)) {
    ictc_set_error("ictc_neighbor_list_noalloc: unsupported box (need cutoff < L/2 and >= 3 cells per axis)%s", "");
    return ICTC_ERR_UNSUPPORTED;
  }
  if (atoms < 0 || atoms > INT32_MAX || !offsets || max_edges < 0 ||
      (atoms > 0 && (!pos || (max_edges > 0 && (!src || !dst || !shift))))) {
    ictc_set_error("ictc_neighbor_list_noalloc: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  const size_t need = workspace_layout(atoms, g.cells(), nullptr, nullptr);
  if (need > kNoAllocScratchBytes) {
    char msg[160];
    snprintf(msg, sizeof(msg), "%zu bytes of cell lists exceed the fixed %zu-byte scratch", need,
             kNoAllocScratchBytes);
    ictc_set_error("ictc_neighbor_list_noalloc: system too large: %s; use ictc_neighbor_count/fill", msg);
    return ICTC_ERR_INVALID;
  }
  void* scratch = nullptr;
  int status = scratch_address((cudaStream_t)stream, &scratch);
  if (status != ICTC_OK) return status;
  status = ictc_neighbor_count(pos, atoms, box, cutoff, scratch, (int64_t)kNoAllocScratchBytes, offsets, stream);
  if (status != ICTC_OK || atoms == 0) return status;
  NeighborWorkspace ws;
  workspace_layout(atoms, g.cells(), &ws, (char*)scratch);
  neighbor_fill_capped_kernel<<<grid_size(atoms, 128), 128, 0, (cudaStream_t)stream>>>(pos, atoms, g, ws, offsets,
                                                                                         max_edges, src, dst, shift);
  return check_launch("ictc_neighbor_list_noalloc: %s");
}
