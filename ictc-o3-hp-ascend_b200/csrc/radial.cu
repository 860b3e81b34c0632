// Fused radial MLP of the MACE interaction on the tensor cores (tcgen05, 3xTF32).
//
// The reference's radial network (mace_ictc/models/pure_cartesian_ictd_fix.py:1545-1553,
// applied per edge at :1787-1800) maps the Bessel x cutoff embedding f [E, F] to the
// per-edge path gates:
//     h1 = s*silu(f W1^T), h2 = s*silu(h1 W2^T), h3 = s*silu(h2 W3^T), gates = h3 W4^T
// with bias-free linears (F -> 64 -> 64 -> 64 -> G) and the normalised SiLU scale s.
//
// radial_forward_kernel: one CTA per SM, tiles of 128 edges; warp-specialised (a
//   control thread issuing MMAs and bulk copies, a hidden-layer warp group and an
//   output warp group); the hidden activations stay on chip and W4 streams from L2.
// radial_w4_adjoint_kernel: dh3 = dgates W4, a streaming GEMM over K = G with a
//   4-stage cp.async pipeline two chunks deep (dgates from HBM, W4^T chunks from L2).
// radial_chain_kernel: recomputes the hidden layers, keeps s*silu'(a_l) in TMEM and
//   runs the chain dh3 -> da3 -> dh2 -> ... -> df.
//
// Every product is 3xTF32 (A_hi B_hi + A_hi B_lo + A_lo B_hi with hi = TF32
// rounding of the value and lo = the FP32 remainder): relative error ~1e-6, the
// FP32 contract of the reference.  Weights arrive pre-split and pre-swizzled in
// one image (ictc_radial_pack) so kernels copy them flat.
#include <cstring>
#include <mutex>

#include "ictc_common.cuh"
#include "ictc_cuda.h"
#include "tc_sm100.cuh"

void ictc_set_error(const char* fmt, const char* detail);

namespace ictc {
namespace {

using namespace tc;

constexpr int kHidden = 64;
constexpr int kMaxFeatures = 8;
constexpr int kTile = 128;             // edges per tile = MMA M
constexpr int kThreads = 512;          // 4 warpgroups; see Slot

// Thread layout: warp w reads TMEM lanes 32*(w % 4) .. +31 (tile rows) and owns the
// column slice w / 4 of every epilogue, so four warps share each row's work.
struct Slot {
  uint32_t row, slice, lane_base;
  __device__ Slot() {
    const uint32_t warp = threadIdx.x / 32;
    row = (warp % 4) * 32 + threadIdx.x % 32;
    slice = warp / 4;
    lane_base = ((warp % 4) * 32) << 16;
  }
};
constexpr float kSiluScale = 1.6791767923989418f;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s: far above any legitimate wait

// Image layout (bytes).  Square hidden weights: hi [2 atoms][64 rows][128 B], lo after.
constexpr uint32_t kSquare = 2 * 2 * kHidden * kAtomBytes;        // 32,768
constexpr uint32_t kW1 = kHidden * kAtomBytes;                    // 8,192: hi k0-7, lo k8-15 per row
constexpr uint32_t kW1T = 2 * 2 * 16 * kAtomBytes;                // 8,192: N = 16 (F padded)
constexpr uint32_t kOffW1 = 0, kOffW2 = kOffW1 + kW1, kOffW3 = kOffW2 + kSquare, kOffW3T = kOffW3 + kSquare,
                   kOffW2T = kOffW3T + kSquare, kOffW1T = kOffW2T + kSquare, kOffW4 = kOffW1T + kW1T;
constexpr uint32_t kHiddenImage = kOffW4;                         // 147,456: W1..W1T

struct RadialShape {
  int features, gates, chunks;
  uint64_t w4, w4t, total;
};

bool radial_shape(int features, int hidden, int gates, RadialShape* s) {
  if (features < 1 || features > kMaxFeatures || hidden != kHidden || gates < 64 || gates % 64) return false;
  s->features = features;
  s->gates = gates;
  s->chunks = gates / 32;
  s->w4 = kOffW4;
  s->w4t = s->w4 + (uint64_t)gates * 512u;
  s->total = s->w4t + (uint64_t)gates * 512u;
  return true;
}

struct RadialArgs {
  const unsigned char* image;
  const float* feats;        // [E, F]
  const float* grad_gates;   // [E, G]
  const float* grad_h3;      // [E, 64]
  float* gates;              // [E, G]
  float* out_h3;             // [E, 64]
  float* grad_feats;         // [E, F]
  int* status;
  int64_t edges;
  int features, gates_width, chunks;
};

__device__ __forceinline__ void flag_error(int* status, int code) {
  if (status) atomicExch(status, code);
}

// Logistic function; the exponent is clamped so 1 + e stays finite.
__device__ __forceinline__ float sigmoid(float a) { return __frcp_rn(1.0f + __expf(fminf(-a, 80.0f))); }
__device__ __forceinline__ float silu_scaled(float a) { return kSiluScale * a * sigmoid(a); }
__device__ __forceinline__ float silu_scaled_grad(float a) {
  const float sig = sigmoid(a);
  return kSiluScale * sig * (1.0f + a * (1.0f - sig));
}

// Flat copy of `bytes` (multiple of 16) from global to shared memory by the block.
__device__ __forceinline__ void copy_flat(unsigned char* dst, const unsigned char* src, uint32_t bytes) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (uint32_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = __ldg(s + i);
}

// Write 16 consecutive K values (k0 .. k0+15, k0 % 16 == 0) of row r into a [128 x 64]
// hi/lo operand (hi atoms at `hi`, lo atoms at hi + 32 KB).
__device__ __forceinline__ void put_operand16(unsigned char* hi, uint32_t r, uint32_t k0, const float* v) {
  const uint32_t atom = k0 / kAtomK, chunk0 = (k0 % kAtomK) / 4;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float4 h, l;
    h.x = tf32_hi(v[4 * q + 0]); l.x = v[4 * q + 0] - h.x;
    h.y = tf32_hi(v[4 * q + 1]); l.y = v[4 * q + 1] - h.y;
    h.z = tf32_hi(v[4 * q + 2]); l.z = v[4 * q + 2] - h.z;
    h.w = tf32_hi(v[4 * q + 3]); l.w = v[4 * q + 3] - h.w;
    const uint32_t off = atom * kTile * kAtomBytes + sw128_chunk(r, chunk0 + q);
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(hi + 2 * kTile * kAtomBytes + off) = l;
  }
}

// Feature row (F <= 8 values) as the layer-1 operand: chunks 0-1 hi, 2-3 lo.
__device__ __forceinline__ void put_features(unsigned char* hbuf, const RadialArgs& a, int64_t e, uint32_t r) {
  float f[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = (e < a.edges && i < a.features) ? __ldg(a.feats + e * a.features + i) : 0.f;
  float hv[8], lv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    hv[i] = tf32_hi(f[i]);
    lv[i] = f[i] - hv[i];
  }
  *reinterpret_cast<float4*>(hbuf + sw128_chunk(r, 0)) = make_float4(hv[0], hv[1], hv[2], hv[3]);
  *reinterpret_cast<float4*>(hbuf + sw128_chunk(r, 1)) = make_float4(hv[4], hv[5], hv[6], hv[7]);
  *reinterpret_cast<float4*>(hbuf + sw128_chunk(r, 2)) = make_float4(lv[0], lv[1], lv[2], lv[3]);
  *reinterpret_cast<float4*>(hbuf + sw128_chunk(r, 3)) = make_float4(lv[4], lv[5], lv[6], lv[7]);
}

// D = A[128 x 64] * B[N x 64]^T for a hi/lo operand at `a` (lo +32 KB) and a weight
// image at `b` with `rows` rows (lo at + 2 * rows * 128).
__device__ __forceinline__ void gemm_k64(uint32_t d, uint32_t a, uint32_t b, uint32_t rows, uint32_t idesc) {
#pragma unroll
  for (uint32_t kk = 0; kk < 8; ++kk) {
    const uint32_t ao = (kk / 4) * kTile * kAtomBytes + (kk % 4) * 32;
    const uint32_t bo = (kk / 4) * rows * kAtomBytes + (kk % 4) * 32;
    mma_tf32x3(d, a + ao, a + 2 * kTile * kAtomBytes + ao, b + bo, b + 2 * rows * kAtomBytes + bo, idesc,
               kk > 0 ? 1u : 0u);
  }
}

// Layer 1 (K = F <= 8 padded to one K step): operand and weights keep hi at
// k 0-7 and lo at k 8-15 of the same rows.
__device__ __forceinline__ void gemm_layer1(uint32_t d, uint32_t a, uint32_t b) {
  mma_tf32x3(d, a, a + 32, b, b + 32, idesc_tf32(kTile, kHidden), 0u);
}

// Block-wide agreement after a wait: every thread learns whether all succeeded.
__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t& phase, int* status) {
  const bool ok = mbar_wait(bar, phase, kWaitNs);
  phase ^= 1u;
  const bool all = __syncthreads_and(ok) != 0;
  if (!all && threadIdx.x == 0) flag_error(status, 1);
  fence_after_sync();
  return all;
}

__device__ __forceinline__ unsigned char* aligned_smem(unsigned char* raw) {
  return reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
}

// ---------------------------------------------------------------------------
// Forward (warp-specialised, activations in TMEM, two MMA issuers)
//
//   warp 0, lane 0  hidden issuer: the three hidden-layer GEMMs of tile i;
//   warp 1, lane 0  output issuer: the W4 chunk GEMMs of tile i-1 and the bulk
//                   copies of W4 chunks;
//   warps 4..11     hidden group: features and s*silu epilogues, written to TMEM;
//   warps 12..19    output group: gate chunks TMEM -> shared staging -> HBM.
// TMEM columns: [0,64) hidden accumulator, [64,192) and [192,320) two activation
// buffers (hi 64 columns, lo 64 columns) used by alternate tiles, [320,336)
// features hi / lo, [384,512) two 64-column gate slots.  A operands are read from
// TMEM, so an MMA only reads its weights from shared memory.  With the activation
// buffers alternating, tile i's hidden chain runs while tile i-1's W4 chunks (and
// their stores) proceed, and the two issuers keep the tensor pipe fed.  W4 chunks
// (32 KB, hi + lo) stream from L2 through a 3-stage shared ring; a stage is
// refilled once the MMAs that read it two chunks earlier are done.
// ---------------------------------------------------------------------------

constexpr int kFwdThreads = 640;
constexpr int kW4Stages = 3, kW4Lag = 2, kD4Slots = 2, kW4Rows = 64;
constexpr uint32_t kW4Chunk = 2 * 2 * kW4Rows * kAtomBytes;  // 32 KB: 64 rows x 64 K, hi + lo
constexpr uint32_t kFwdW4 = kOffW3T;                         // W4 ring after W1, W2, W3
constexpr uint32_t kStageRow = kW4Rows * 4 + 16;             // padded row of the output staging
constexpr uint32_t kFwdOut = kFwdW4 + kW4Stages * kW4Chunk;  // gate chunk staging [128][kStageRow]
constexpr uint32_t kFwdBar = kFwdOut + kTile * kStageRow;
constexpr uint32_t kFwdSmem = kFwdBar + 256 + 1024;
constexpr uint32_t kColH0 = 64, kColHStep = 128, kColF = 320, kColFLo = 328, kColOut = 384;

struct FwdBars {
  uint64_t op_ready, acc_full, h3_ready[2], h_free[2];
  uint64_t w4_full[kW4Stages], w4_empty[kW4Stages];
  uint64_t d4_full[kD4Slots], d4_empty[kD4Slots];
  uint32_t tmem_slot;
  int abort;
};

// D = A[TMEM, 128 x 64 hi/lo] * B[smem image, rows x 64]^T.
__device__ __forceinline__ void gemm_k64_ta(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t b, uint32_t rows,
                                            uint32_t idesc) {
#pragma unroll
  for (uint32_t kk = 0; kk < 8; ++kk) {
    const uint32_t bo = (kk / 4) * rows * kAtomBytes + (kk % 4) * 32;
    mma_tf32x3_ta(d, a_hi + 8 * kk, a_lo + 8 * kk, b + bo, b + 2 * rows * kAtomBytes + bo, idesc,
                  kk > 0 ? 1u : 0u);
  }
}

__global__ void __launch_bounds__(kFwdThreads, 1) radial_forward_kernel(RadialArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = aligned_smem(smem_raw);
  FwdBars* b = reinterpret_cast<FwdBars*>(smem + kFwdBar);
  volatile int* abort = &b->abort;
  const uint32_t warp = threadIdx.x / 32;
  const int chunks = a.gates_width / kW4Rows;
  const int64_t tiles = (a.edges + kTile - 1) / kTile;
  const int64_t my_tiles = tiles > blockIdx.x ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  copy_flat(smem, a.image, kOffW3T);                 // W1, W2, W3
  if (threadIdx.x == 0) {
    mbar_init(&b->op_ready, 1);
    mbar_init(&b->acc_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b->h3_ready[i], 1);
      mbar_init(&b->h_free[i], 1);
    }
    for (int i = 0; i < kW4Stages; ++i) {
      mbar_init(&b->w4_full[i], 1);
      mbar_init(&b->w4_empty[i], 1);
    }
    for (int i = 0; i < kD4Slots; ++i) {
      mbar_init(&b->d4_full[i], 1);
      mbar_init(&b->d4_empty[i], 8);
    }
    b->abort = 0;
  }
  if (warp == 0) tmem_alloc(&b->tmem_slot, 512);
  fence_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = b->tmem_slot;
  const uint32_t base = smem_u32(smem);
  const unsigned char* w4_image = a.image + kOffW4;
  const uint32_t id64 = idesc_tf32(kTile, kHidden);

  if (threadIdx.x == 0) {
    // ----- hidden issuer -----
    uint32_t op_phase = 0;
    bool ok = true;
    auto wait_op = [&]() {
      ok = ok && mbar_wait_or_abort(&b->op_ready, op_phase, kWaitNs, abort);
      op_phase ^= 1u;
      fence_after_sync();
      return ok;
    };
    for (int64_t i = 0; i < my_tiles && ok; ++i) {
      const uint32_t h = tmem + kColH0 + kColHStep * (uint32_t)(i & 1);
      if (!wait_op()) break;                         // features in TMEM
      mma_tf32x3_ta(tmem, tmem + kColF, tmem + kColFLo, base + kOffW1, base + kOffW1 + 32, id64, 0u);
      mma_commit(&b->acc_full);
      for (int layer = 0; layer < 2 && ok; ++layer) {
        if (!wait_op()) break;                       // h1, h2 in this tile's buffer
        gemm_k64_ta(tmem, h, h + 64, base + (layer == 0 ? kOffW2 : kOffW3), kHidden, id64);
        mma_commit(&b->acc_full);
      }
    }
    // The hidden group consumes the last acc_full only after that MMA completed.
  } else if (threadIdx.x == 32) {
    // ----- output issuer -----
    uint32_t h3_phase[2] = {}, full_phase[kW4Stages] = {}, empty_phase[kW4Stages] = {}, d4e_phase[kD4Slots] = {};
    int64_t wcount = 0, issued = 0;
    const int64_t total_chunks = my_tiles * chunks;
    auto request = [&](int64_t n) {
      const int st = (int)(n % kW4Stages);
      mbar_arrive_expect(&b->w4_full[st], kW4Chunk);
      bulk_load(smem + kFwdW4 + st * kW4Chunk, w4_image + (uint64_t)(n % chunks) * kW4Chunk, kW4Chunk,
                &b->w4_full[st]);
    };
    for (; issued < total_chunks && issued < kW4Stages - kW4Lag; ++issued) request(issued);
    bool ok = true;
    int64_t i = 0;
    for (; i < my_tiles && ok; ++i) {
      const uint32_t buf = (uint32_t)(i & 1);
      const uint32_t h = tmem + kColH0 + kColHStep * buf;
      ok = mbar_wait_or_abort(&b->h3_ready[buf], h3_phase[buf], kWaitNs, abort);
      h3_phase[buf] ^= 1u;
      if (!ok) break;
      for (int j = 0; j < chunks && ok; ++j, ++wcount) {
        const int st = (int)(wcount % kW4Stages), slot = (int)(wcount % kD4Slots);
        if (issued < total_chunks) {                 // refill the stage read kW4Lag chunks ago
          const int fs = (int)(issued % kW4Stages);
          if (issued >= kW4Stages) {
            ok = mbar_wait_or_abort(&b->w4_empty[fs], empty_phase[fs], kWaitNs, abort);
            empty_phase[fs] ^= 1u;
            if (!ok) break;
          }
          request(issued++);
        }
        ok = mbar_wait_or_abort(&b->w4_full[st], full_phase[st], kWaitNs, abort);
        full_phase[st] ^= 1u;
        if (ok && wcount >= kD4Slots) {
          ok = mbar_wait_or_abort(&b->d4_empty[slot], d4e_phase[slot], kWaitNs, abort);
          d4e_phase[slot] ^= 1u;
        }
        if (!ok) break;
        fence_after_sync();
        gemm_k64_ta(tmem + kColOut + kW4Rows * slot, h, h + 64, base + kFwdW4 + st * kW4Chunk, kW4Rows,
                    idesc_tf32(kTile, kW4Rows));
        mma_commit(&b->d4_full[slot]);
        mma_commit(&b->w4_empty[st]);
      }
      mma_commit(&b->h_free[buf]);                   // this buffer may be overwritten once these finish
    }
    // Wait (bounded) for the last commit so every MMA of this issuer is complete.
    if (i > 0) mbar_wait(&b->h_free[(i - 1) & 1], (uint32_t)(((i - 1) >> 1) & 1), kWaitNs);
  } else if (warp >= 4 && warp < 12) {
    // ----- hidden group: 8 warps, quadrant warp % 4, column half (warp - 4) / 4 -----
    const uint32_t row = (warp % 4) * 32 + threadIdx.x % 32;
    const uint32_t half = (warp - 4) / 4;
    const uint32_t lanes = tmem + (((warp % 4) * 32) << 16);
    uint32_t acc_phase = 0, hfree_phase[2] = {};
    bool ok = true;
    int64_t count = 0;
    for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++count) {
      const int64_t e = t * kTile + row;
      const uint32_t buf = (uint32_t)(count & 1);
      const uint32_t hcol = kColH0 + kColHStep * buf;
      if (half == 0) {
        float f[8], hi[8], lo[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          f[i] = (e < a.edges && i < a.features) ? __ldg(a.feats + e * a.features + i) : 0.f;
          hi[i] = tf32_hi(f[i]);
          lo[i] = f[i] - hi[i];
        }
        tmem_store8(lanes + kColF, hi);
        tmem_store8(lanes + kColFLo, lo);
      }
      fence_before_sync();
      named_barrier(1, 256);
      if (threadIdx.x == 128) mbar_arrive(&b->op_ready);
      for (int layer = 0; layer < 3 && ok; ++layer) {
        ok = named_barrier_all(1, 256, mbar_wait_or_abort(&b->acc_full, acc_phase, kWaitNs, abort));
        acc_phase ^= 1u;
        if (!ok) break;
        if (layer == 0 && count >= 2) {              // tile count-2's W4 MMAs still read this buffer
          ok = named_barrier_all(1, 256, mbar_wait_or_abort(&b->h_free[buf], hfree_phase[buf], kWaitNs, abort));
          hfree_phase[buf] ^= 1u;
          if (!ok) break;
        }
        fence_after_sync();
        float v[32], hi[16], lo[16];
        tmem_load16(lanes + 32 * half, v);
        tmem_load16(lanes + 32 * half + 16, v + 16);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float h = silu_scaled(v[16 * q + i]);
            hi[i] = tf32_hi(h);
            lo[i] = h - hi[i];
          }
          tmem_store16_async(lanes + hcol + 32 * half + 16 * q, hi);
          tmem_store16_async(lanes + hcol + 64 + 32 * half + 16 * q, lo);
        }
        tmem_store_wait();
        fence_before_sync();
        named_barrier(1, 256);
        if (threadIdx.x == 128) mbar_arrive(layer < 2 ? &b->op_ready : &b->h3_ready[buf]);
      }
    }
  } else if (warp >= 12) {
    // ----- output group: 8 warps, quadrant warp % 4, 32-column half of each chunk -----
    const uint32_t row = (warp % 4) * 32 + threadIdx.x % 32;
    const uint32_t half = (warp - 12) / 4;
    const uint32_t lanes = tmem + (((warp % 4) * 32) << 16);
    uint32_t full_phase[kD4Slots] = {};
    int64_t wcount = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      for (int j = 0; j < chunks; ++j, ++wcount) {
        const int slot = (int)(wcount % kD4Slots);
        // Group-wide: all reads of the previous chunk's staging are done, and all agree on ok.
        ok = named_barrier_all(2, 256, mbar_wait_or_abort(&b->d4_full[slot], full_phase[slot], kWaitNs, abort));
        full_phase[slot] ^= 1u;
        if (!ok) break;
        fence_after_sync();
        float v[32];
        tmem_load16(lanes + kColOut + kW4Rows * slot + 32 * half, v);
        tmem_load16(lanes + kColOut + kW4Rows * slot + 32 * half + 16, v + 16);
        fence_before_sync();
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&b->d4_empty[slot]);
        float4* stage_row = reinterpret_cast<float4*>(smem + kFwdOut + row * kStageRow + 128 * half);
#pragma unroll
        for (int q = 0; q < 8; ++q) stage_row[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        named_barrier(2, 256);
        // 128 rows x 16 float4: 16 consecutive threads write one row's 256 contiguous bytes.
        const uint32_t ot = threadIdx.x - 384;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t idx = ot + 256 * q, r = idx / 16, c4 = idx % 16;
          const int64_t er = t * kTile + r;
          const float4 val = *reinterpret_cast<const float4*>(smem + kFwdOut + r * kStageRow + 16 * c4);
          if (er < a.edges)
            *reinterpret_cast<float4*>(a.gates + er * a.gates_width + kW4Rows * j + 4 * c4) = val;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && *abort) flag_error(a.status, 4);
  if (warp == 0) {
    __syncwarp();
    fence_after_sync();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// dh3 = dgates W4 (K = G streamed in chunks of 32)
// ---------------------------------------------------------------------------

constexpr int kStages = 4;
constexpr uint32_t kStageBytes = 3 * 16384;  // A hi, A lo, B (W4^T chunk hi+lo)
// K chunks rotate over independent TMEM accumulators, summed in FP32 at the end:
// the tensor core's accumulation error grows with the K it sums, and G reaches
// thousands.
constexpr int kAccumulators = 4;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Warp-specialised: warp 0 lane 0 issues the MMAs; warps 4..19 (the workers, two
// groups taking alternate K chunks) load dgates rows and W4^T chunks with
// cp.async, split dgates into hi/lo in place, and write dh3.  Two sets of kAccumulators TMEM accumulators alternate between tiles
// so a tile's MMAs can start while the previous tile's dh3 is written.
constexpr int kAdjThreads = 640;

struct AdjBars {
  uint64_t split_done[kStages], mma_done[kStages], acc_full[2], acc_free[2];
  uint32_t tmem_slot;
  int abort;
};

__global__ void __launch_bounds__(kAdjThreads, 1) radial_w4_adjoint_kernel(RadialArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = aligned_smem(smem_raw);
  AdjBars* b = reinterpret_cast<AdjBars*>(smem + kStages * kStageBytes);
  volatile int* abort = &b->abort;
  const uint32_t warp = threadIdx.x / 32;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&b->split_done[i], 1);
      mbar_init(&b->mma_done[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b->acc_full[i], 1);
      mbar_init(&b->acc_free[i], 1);
    }
    b->abort = 0;
  }
  if (warp == 0) tmem_alloc(&b->tmem_slot, 512);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = b->tmem_slot;
  const uint32_t base = smem_u32(smem);
  const int64_t tiles = (a.edges + kTile - 1) / kTile;
  const int chunks = a.chunks;
  const int used = chunks < kAccumulators ? chunks : kAccumulators;
  const int64_t my_tiles = tiles > blockIdx.x ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t total = my_tiles * chunks;
  auto item_tile = [&](int64_t q) { return blockIdx.x + (q / chunks) * gridDim.x; };

  if (warp == 0) {
    if (threadIdx.x == 0) {
      // ----- MMA issue -----
      uint32_t split_phase[kStages] = {}, free_phase[2] = {};
      bool ok = true;
      for (int64_t q = 0; q < total && ok; ++q) {
        const int s = (int)(q % kStages), chunk = (int)(q % chunks);
        const int64_t ti = q / chunks;
        const uint32_t buf = (uint32_t)(ti & 1);
        if (chunk == 0 && ti >= 2) {
          ok = mbar_wait_or_abort(&b->acc_free[buf], free_phase[buf], kWaitNs, abort);
          free_phase[buf] ^= 1u;
          if (!ok) break;
        }
        ok = mbar_wait_or_abort(&b->split_done[s], split_phase[s], kWaitNs, abort);
        split_phase[s] ^= 1u;
        if (!ok) break;
        fence_after_sync();
        const uint32_t sa = base + s * kStageBytes;
        const uint32_t acc = tmem + 256 * buf + 64 * (chunk % kAccumulators);
#pragma unroll
        for (uint32_t kk = 0; kk < 4; ++kk)
          mma_tf32x3(acc, sa + kk * 32, sa + 16384 + kk * 32, sa + 32768 + kk * 32, sa + 32768 + 8192 + kk * 32,
                     idesc_tf32(kTile, kHidden), (chunk >= kAccumulators || kk > 0) ? 1u : 0u);
        mma_commit(&b->mma_done[s]);
        if (chunk == chunks - 1) mma_commit(&b->acc_full[buf]);
      }
    }
  } else if (warp >= 4) {
    // ----- workers: two groups of 8 warps; group g handles items q = g, g + 2, ... in
    // stages g, g + 2 (q % 4), one item ahead.  Epilogue slot: quadrant warp % 4,
    // 32-column half ((warp - 4) / 4) % 2. -----
    const uint32_t grp = (warp - 4) / 8;
    const uint32_t gt = threadIdx.x - 128 - 256 * grp;   // 0 .. 255 within the group
    const uint32_t bar_id = 1 + grp;
    const uint32_t row = (warp % 4) * 32 + threadIdx.x % 32;
    const uint32_t half = ((warp - 4) / 4) % 2;
    const uint32_t lanes = tmem + (((warp % 4) * 32) << 16);
    uint32_t done_phase[kStages] = {}, full_phase[2] = {};
    bool ok = true;
    auto issue = [&](int64_t q) {
      const uint32_t stage = base + (uint32_t)(q % kStages) * kStageBytes;
      const int64_t tile = item_tile(q);
      const int chunk = (int)(q % chunks);
#pragma unroll
      for (int i = 0; i < 1024 / 256; ++i) {
        const uint32_t idx = gt + 256 * i;
        const uint32_t r = idx / 8, ch = idx % 8;
        const int64_t e = tile * kTile + r;
        const bool valid = e < a.edges;
        const float* src = valid ? a.grad_gates + e * a.gates_width + chunk * 32 + ch * 4 : a.grad_gates;
        cp_async16(stage + sw128_chunk(r, ch), src, valid ? 16u : 0u);
      }
      const unsigned char* img = a.image + kOffW4 + (uint64_t)a.gates_width * 512u + (uint64_t)chunk * 16384u;
#pragma unroll
      for (int i = 0; i < 1024 / 256; ++i) {
        const uint32_t idx = gt + 256 * i;
        cp_async16(stage + 2 * 16384 + idx * 16, img + idx * 16, 16u);
      }
    };
    if ((int64_t)grp < total) issue(grp);
    cp_async_commit();
    for (int64_t q = grp; q < total && ok; q += 2) {
      const int s = (int)(q % kStages), chunk = (int)(q % chunks);
      const int64_t next = q + 2;                    // same group, the other stage of the group
      if (next < total) {
        if (next >= kStages) {                       // that stage last held item next - 4
          const int ns = (int)(next % kStages);
          ok = named_barrier_all(bar_id, 256, mbar_wait_or_abort(&b->mma_done[ns], done_phase[ns], kWaitNs, abort));
          done_phase[ns] ^= 1u;
          if (!ok) break;
        }
        issue(next);
      }
      cp_async_commit();
      cp_async_wait<1>();
      named_barrier(bar_id, 256);
      unsigned char* st = smem + s * kStageBytes;
#pragma unroll
      for (int i = 0; i < 1024 / 256; ++i) {
        const uint32_t off = (gt + 256 * i) * 16;
        float4 v = *reinterpret_cast<float4*>(st + off);
        float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
        *reinterpret_cast<float4*>(st + off) = h;
        *reinterpret_cast<float4*>(st + 16384 + off) = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
      }
      fence_async_smem();
      named_barrier(bar_id, 256);
      if (gt == 0) mbar_arrive(&b->split_done[s]);
      if (chunk == chunks - 1) {
        const int64_t ti = q / chunks;
        const uint32_t buf = (uint32_t)(ti & 1);
        ok = named_barrier_all(bar_id, 256,
                               mbar_wait_or_abort(&b->acc_full[buf], full_phase[buf], kWaitNs, abort));
        full_phase[buf] ^= 1u;
        if (!ok) break;
        fence_after_sync();
        const int64_t e = item_tile(q) * kTile + row;
        float v[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_load16(lanes + 256 * buf + 32 * half + 16 * c, v + 16 * c);
          for (int j = 1; j < used; ++j) {
            float w[16];
            tmem_load16(lanes + 256 * buf + 64 * j + 32 * half + 16 * c, w);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[16 * c + i] += w[i];
          }
        }
        fence_before_sync();
        named_barrier(bar_id, 256);
        if (gt == 0) mbar_arrive(&b->acc_free[buf]);
        if (e < a.edges) {
          float4* dst = reinterpret_cast<float4*>(a.out_h3 + e * kHidden + 32 * half);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) dst[q4] = make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
        }
      }
    }
    cp_async_wait<0>();
  }
  __syncthreads();
  if (threadIdx.x == 0 && *abort) flag_error(a.status, 5);
  if (warp == 0) {
    if (threadIdx.x == 0 && *abort) {
      // After an error, MMAs may still be in flight: wait (bounded) for the last one issued.
      for (int i = 0; i < kStages; ++i) mbar_wait(&b->mma_done[i], 0, 1000000ull);
    }
    __syncwarp();
    fence_after_sync();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Chain: recompute a1..a3, then dh3 -> df
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kThreads, 1) radial_chain_kernel(RadialArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = aligned_smem(smem_raw);
  constexpr uint32_t kSH = kHiddenImage;             // 147,456
  constexpr uint32_t kSBar = kSH + 65536;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kSBar);
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + kSBar + 8);
  copy_flat(smem, a.image, kHiddenImage);
  if (threadIdx.x == 0) mbar_init(bar, 1);
  if (threadIdx.x < 32) tmem_alloc(slot, 256);
  fence_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *slot;
  const Slot me;
  const uint32_t r = me.row;
  const uint32_t base = smem_u32(smem);
  const uint32_t trow = tmem + me.lane_base;
  const uint32_t col = 16 * me.slice;                // this thread's 16 columns
  uint32_t phase = 0;
  const int64_t tiles = (a.edges + kTile - 1) / kTile;
  const uint32_t id64 = idesc_tf32(kTile, kHidden);
  bool ok = true;

  auto issue = [&](auto&& body) {
    fence_async_smem();
    fence_before_sync();
    __syncthreads();
    if (threadIdx.x == 0) {
      fence_after_sync();
      body();
      mma_commit(bar);
    }
  };

  for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
    const int64_t e = t * kTile + r;
    if (me.slice == 0) put_features(smem + kSH, a, e, r);
    issue([&] { gemm_layer1(tmem, base + kSH, base + kOffW1); });
    ok = wait_all(bar, phase, a.status);
    // Forward recompute: keep s*silu'(a_l) in TMEM columns 64 + 64*l.
    for (int layer = 0; ok && layer < 3; ++layer) {
      float v[16], d[16];
      tmem_load16(trow + col, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        d[i] = silu_scaled_grad(v[i]);
        v[i] = silu_scaled(v[i]);
      }
      tmem_store16(trow + 64 + 64 * layer + col, d);
      if (layer < 2) {
        put_operand16(smem + kSH, r, col, v);
        issue([&] { gemm_k64(tmem, base + kSH, base + (layer == 0 ? kOffW2 : kOffW3), kHidden, id64); });
        ok = wait_all(bar, phase, a.status);
      }
    }
    if (!ok) break;
    // da3 = dh3 * s*silu'(a3)
    {
      float v[16], d[16];
      tmem_load16(trow + 192 + col, d);
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        float4 g = e < a.edges ? __ldg(reinterpret_cast<const float4*>(a.grad_h3 + e * kHidden + col + i))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        v[i] = g.x * d[i];
        v[i + 1] = g.y * d[i + 1];
        v[i + 2] = g.z * d[i + 2];
        v[i + 3] = g.w * d[i + 3];
      }
      put_operand16(smem + kSH, r, col, v);
    }
    // dh2 = da3 W3, da2 = dh2 * s2; dh1 = da2 W2, da1 = dh1 * s1.
    for (int layer = 1; ok && layer >= 0; --layer) {
      issue([&] { gemm_k64(tmem, base + kSH, base + (layer == 1 ? kOffW3T : kOffW2T), kHidden, id64); });
      ok = wait_all(bar, phase, a.status);
      if (!ok) break;
      float v[16], d[16];
      tmem_load16(trow + col, v);
      tmem_load16(trow + 64 + 64 * layer + col, d);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] *= d[i];
      put_operand16(smem + kSH, r, col, v);
    }
    if (!ok) break;
    // df = da1 W1 (N = 16, columns >= F are zero).
    issue([&] { gemm_k64(tmem, base + kSH, base + kOffW1T, 16, idesc_tf32(kTile, 16)); });
    ok = wait_all(bar, phase, a.status);
    if (!ok) break;
    if (me.slice == 0) {
      float v[16];
      tmem_load16(trow, v);
      if (e < a.edges)
        for (int i = 0; i < a.features; ++i) a.grad_feats[e * a.features + i] = v[i];
    }
    fence_before_sync();
    __syncthreads();
  }
  if (!ok) mbar_wait(bar, phase, kWaitNs);
  fence_before_sync();
  __syncthreads();
  if (threadIdx.x < 32) {
    fence_after_sync();
    tmem_dealloc(tmem, 256);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

constexpr uint32_t kAdjointSmem = kStages * kStageBytes + 256 + 1024;
static_assert(sizeof(AdjBars) <= 256, "adjoint barrier block");
constexpr uint32_t kChainSmem = kHiddenImage + 65536 + 64 + 1024;

int sm_count() {
  int device = 0, sms = 0;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  return sms > 0 ? sms : 1;
}

template <class K>
int prepare_kernel(K kernel, uint32_t smem) {
  // Per-device attribute: set on every call (cheap) so multi-GPU processes are covered.
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) {
    ictc_set_error("radial MLP: %s", cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}

static_assert(kFwdSmem <= 232448, "forward shared memory");
static_assert(sizeof(FwdBars) <= 256, "forward barrier block");
static_assert(kFwdBar % 8 == 0, "barrier alignment");

int launch_forward(const RadialArgs& a, cudaStream_t s) {
  if (int st = prepare_kernel(radial_forward_kernel, kFwdSmem)) return st;
  const int64_t tiles = (a.edges + kTile - 1) / kTile;
  const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
  radial_forward_kernel<<<grid, kFwdThreads, kFwdSmem, s>>>(a);
  return ICTC_OK;
}

// Host copy of the 3xTF32 split.
void split(float x, float* hi, float* lo) {
  uint32_t bits;
  std::memcpy(&bits, &x, 4);
  bits = tf32_round_bits(bits);
  std::memcpy(hi, &bits, 4);
  *lo = x - *hi;
}

void put(unsigned char* img, uint32_t off, float v) { std::memcpy(img + off, &v, 4); }

// K-major hi/lo image of B[n][k] (rows x 64), hi atoms then lo atoms.
template <class F>
void pack_square(unsigned char* img, uint32_t rows, F value) {
  for (uint32_t n = 0; n < rows; ++n)
    for (uint32_t k = 0; k < (uint32_t)kHidden; ++k) {
      float hi, lo;
      split(value(n, k), &hi, &lo);
      put(img, sw128_offset(rows, n, k), hi);
      put(img, 2 * rows * kAtomBytes + sw128_offset(rows, n, k), lo);
    }
}

}  // namespace
}  // namespace ictc

using namespace ictc;

extern "C" int64_t ictc_radial_image_bytes(int features, int hidden, int gates) {
  RadialShape s;
  if (!radial_shape(features, hidden, gates, &s)) return -1;
  return (int64_t)s.total;
}

extern "C" int ictc_radial_pack(const float* w1, const float* w2, const float* w3, const float* w4, int features,
                                int hidden, int gates, void* image, int64_t image_bytes) {
  RadialShape s;
  if (!radial_shape(features, hidden, gates, &s)) {
    ictc_set_error("ictc_radial_pack: unsupported shape (F <= 8, hidden 64, gates a multiple of 64)%s", "");
    return ICTC_ERR_UNSUPPORTED;
  }
  if (!w1 || !w2 || !w3 || !w4 || !image || image_bytes < (int64_t)s.total) {
    ictc_set_error("ictc_radial_pack: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  unsigned char* img = static_cast<unsigned char*>(image);
  std::memset(img, 0, s.total);
  const int F = features, H = kHidden;
  // W1 [64, F]: hi at k 0-7, lo at k 8-15 of each row.
  for (int n = 0; n < H; ++n)
    for (int k = 0; k < F; ++k) {
      float hi, lo;
      split(w1[n * F + k], &hi, &lo);
      put(img + kOffW1, sw128_offset(H, n, k), hi);
      put(img + kOffW1, sw128_offset(H, n, 8 + k), lo);
    }
  pack_square(img + kOffW2, H, [&](uint32_t n, uint32_t k) { return w2[n * H + k]; });
  pack_square(img + kOffW3, H, [&](uint32_t n, uint32_t k) { return w3[n * H + k]; });
  pack_square(img + kOffW3T, H, [&](uint32_t n, uint32_t k) { return w3[k * H + n]; });
  pack_square(img + kOffW2T, H, [&](uint32_t n, uint32_t k) { return w2[k * H + n]; });
  pack_square(img + kOffW1T, 16, [&](uint32_t n, uint32_t k) { return (int)n < F ? w1[k * F + n] : 0.f; });
  // W4 [G, 64] for the forward in chunks of 64 rows (32 KB each).
  for (int c = 0; c < gates / kW4Rows; ++c)
    pack_square(img + s.w4 + (uint64_t)c * kW4Chunk, kW4Rows,
                [&](uint32_t n, uint32_t k) { return w4[(uint64_t)(kW4Rows * c + n) * H + k]; });
  // W4^T chunks for the adjoint: chunk c = rows n (64) x k in [32c, 32c+32).
  for (int c = 0; c < s.chunks; ++c) {
    unsigned char* chunk = img + s.w4t + (uint64_t)c * 16384;
    for (int n = 0; n < H; ++n)
      for (int k = 0; k < 32; ++k) {
        float hi, lo;
        split(w4[(uint64_t)(32 * c + k) * H + n], &hi, &lo);
        put(chunk, sw128_offset(H, n, k), hi);
        put(chunk + 8192, sw128_offset(H, n, k), lo);
      }
  }
  return ICTC_OK;
}

extern "C" int ictc_radial_forward(const void* image, const float* feats, float* gates, int64_t edges,
                                   int features, int hidden, int gates_width, int* status, void* stream) {
  RadialShape s;
  if (!radial_shape(features, hidden, gates_width, &s)) {
    ictc_set_error("ictc_radial_forward: unsupported shape%s", "");
    return ICTC_ERR_UNSUPPORTED;
  }
  if (edges < 0 || (edges > 0 && (!image || !feats || !gates))) {
    ictc_set_error("ictc_radial_forward: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  if (edges == 0) return ICTC_OK;
  RadialArgs a{};
  a.image = static_cast<const unsigned char*>(image);
  a.feats = feats;
  a.gates = gates;
  a.status = status;
  a.edges = edges;
  a.features = features;
  a.gates_width = gates_width;
  a.chunks = s.chunks;
  cudaStream_t st = (cudaStream_t)stream;
  const int rc = launch_forward(a, st);
  if (rc) return rc;
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error("ictc_radial_forward: %s", cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}

extern "C" int ictc_radial_backward(const void* image, const float* feats, const float* grad_gates,
                                    float* grad_h3, float* grad_feats, int64_t edges, int features, int hidden,
                                    int gates_width, int* status, void* stream) {
  RadialShape s;
  if (!radial_shape(features, hidden, gates_width, &s)) {
    ictc_set_error("ictc_radial_backward: unsupported shape%s", "");
    return ICTC_ERR_UNSUPPORTED;
  }
  if (edges < 0 || (edges > 0 && (!image || !feats || !grad_gates || !grad_h3 || !grad_feats))) {
    ictc_set_error("ictc_radial_backward: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  if (edges == 0) return ICTC_OK;
  RadialArgs a{};
  a.image = static_cast<const unsigned char*>(image);
  a.feats = feats;
  a.grad_gates = grad_gates;
  a.grad_h3 = grad_h3;
  a.out_h3 = grad_h3;
  a.grad_feats = grad_feats;
  a.status = status;
  a.edges = edges;
  a.features = features;
  a.gates_width = gates_width;
  a.chunks = s.chunks;
  cudaStream_t st = (cudaStream_t)stream;
  if (int rc = prepare_kernel(radial_w4_adjoint_kernel, kAdjointSmem)) return rc;
  if (int rc = prepare_kernel(radial_chain_kernel, kChainSmem)) return rc;
  const int64_t tiles = (edges + kTile - 1) / kTile;
  const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
  radial_w4_adjoint_kernel<<<grid, kAdjThreads, kAdjointSmem, st>>>(a);
  radial_chain_kernel<<<grid, kThreads, kChainSmem, st>>>(a);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error("ictc_radial_backward: %s", cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}

// ---------------------------------------------------------------------------
// Self-test of the bounded waits (failure detection without a GPU fault)
// ---------------------------------------------------------------------------

namespace ictc {
namespace {

// One CTA waits on an mbarrier that nothing ever arrives on: the wait must give
// up after `limit_ns`, record the failure in *status and return normally, leaving
// the context usable.  `arrive` = 1 makes one thread arrive first (the success path).
__global__ void wait_selftest_kernel(int* status, uint64_t limit_ns, int arrive) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    abort_flag = 0;
  }
  __syncthreads();
  if (arrive && threadIdx.x == 0) tc::mbar_arrive(&bar);
  const bool ok = tc::mbar_wait_or_abort(&bar, 0, limit_ns, &abort_flag);
  const bool all = __syncthreads_and(ok) != 0;
  if (threadIdx.x == 0) *status = all ? 0 : 1;
}

}  // namespace
}  // namespace ictc

extern "C" int ictc_wait_selftest(int* status, int64_t limit_ns, int arrive, void* stream) {
  if (!status || limit_ns <= 0 || limit_ns > 5000000000ll) {
    ictc_set_error("ictc_wait_selftest: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  ictc::wait_selftest_kernel<<<1, 64, 0, (cudaStream_t)stream>>>(status, (uint64_t)limit_ns, arrive);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error("ictc_wait_selftest: %s", cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}
