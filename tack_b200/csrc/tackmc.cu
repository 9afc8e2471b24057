// tackmc.cu -- sm_100a kernels and C ABI of libtackmc.so.
//
// Flying edges (merged-point marching cubes) over a uniform f32 volume, in
// three device passes and one small host round trip:
//
//   K1 fe_threshold  one streaming read of the volume; every node becomes one
//                    bit per isovalue ("value > isovalue", NaN -> 0) in a flat
//                    bitmask, 1/32 of the volume's size.
//   K2 fe_count_scan per node row: popcounts of x/y/z edge crossings and the
//                    triangle count of the cell row, from the bitmask only;
//                    a single-pass decoupled look-back scan turns them into
//                    exact per-row offsets; rows with any output go to a
//                    worklist.
//   (host)           counts -> allocate outputs of the exact size.
//   K3 fe_emit       active rows only: point ids are popcount ranks in the
//                    bitmask; node values are read only at crossing edges.
//
// The arithmetic of an emitted point is the reference's, operation for
// operation, in IEEE f32 without contraction (flying_edges.py:480-542):
//   t = (iso - s) / ((s1 - s) + 1e-10f);  p = p0 + t * (p1 - p0),
//   p0 = x0 + float(i) * dx.
// Output ordering is the reference's (flying_edges.py:545-656), so points and
// connectivity are identical, not just equivalent.
//
// Nothing here is a dense contraction; every kernel is bounded by HBM or
// latency, so there are no tensor-core paths.  Device-side waits (look-back)
// are bounded by %globaltimer and report TKMC_ERR_DEVICE_TIMEOUT.

#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "mc_tables.h"
#include "tackmc.h"

#define TKMC_VERSION 100

namespace {

// ------------------------------------------------------------------------
// host-side state and error handling
// ------------------------------------------------------------------------

thread_local char g_err[512] = "";
std::atomic<uint64_t> g_launches{0};
std::atomic<int64_t> g_wait_ns{1000000000LL};
std::atomic<int64_t> g_skip_tile{-1};

int set_err(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

#define TK_CUDA(call)                                                        \
  do {                                                                       \
    cudaError_t e_ = (call);                                                 \
    if (e_ != cudaSuccess)                                                   \
      return set_err(TKMC_ERR_CUDA, "%s failed: %s", #call,                  \
                     cudaGetErrorString(e_));                                \
  } while (0)

#define TK_LAUNCHED()                                                        \
  do {                                                                       \
    g_launches.fetch_add(1, std::memory_order_relaxed);                      \
    cudaError_t e_ = cudaGetLastError();                                     \
    if (e_ != cudaSuccess)                                                   \
      return set_err(TKMC_ERR_CUDA, "kernel launch failed: %s",              \
                     cudaGetErrorString(e_));                                \
  } while (0)

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) !=
            cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ------------------------------------------------------------------------
// device helpers
// ------------------------------------------------------------------------

#define TKMC_PACK_CASE(s) tkmc::pack_case(s),
// Packed case table: nibbles 0..14 edge ids, nibble 15 triangle count.
__constant__ uint64_t c_case_tris[256] = {TKMC_CASE_LIST(TKMC_PACK_CASE)};
#undef TKMC_PACK_CASE

constexpr int kThreads = 256;
constexpr int kRowsPerTile = 256;  // K2 tile: one row per thread in the scan
constexpr int kScanItems = 16;     // generic scan: items per thread
constexpr int kScanTile = kThreads * kScanItems;

struct IsoParams {
  float v[TKMC_MAX_ISO];
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bits [0, n) set; n clamped to [0, 32].
__device__ __forceinline__ uint32_t low_mask(int n) {
  return n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : ((1u << n) - 1u));
}

// (x >> 1) with bit 31 taken from bit 0 of the next word.
__device__ __forceinline__ uint32_t shr1(uint32_t x, uint32_t next) {
  return __funnelshift_r(x, next, 1);
}

// Nodes [32w, 32w+32) of the row whose first node is flat bit `rowbit`,
// zero beyond the row's length L.
__device__ __forceinline__ uint32_t row_word(const uint32_t* __restrict__ bits,
                                             int64_t rowbit, int w, int64_t L) {
  const int64_t rem = L - 32 * (int64_t)w;
  if (rem <= 0) return 0u;
  const int64_t pos = rowbit + 32 * (int64_t)w;
  const int64_t q = pos >> 5;
  const int sh = (int)(pos & 31);
  uint32_t x = __ldg(bits + q);
  if (sh) x = __funnelshift_r(x, __ldg(bits + q + 1), sh);
  if (rem < 32) x &= (1u << rem) - 1u;
  return x;
}

// Exact f32 point arithmetic of the reference (no contraction).
__device__ __forceinline__ float coord(float o, int64_t i, float h) {
  return __fadd_rn(o, __fmul_rn(__ll2float_rn((long long)i), h));
}
__device__ __forceinline__ float lerp_ref(float p0, float p1, float t) {
  return __fadd_rn(p0, __fmul_rn(t, __fsub_rn(p1, p0)));
}
__device__ __forceinline__ float interp_t(float iso, float s, float s1) {
  return __fdiv_rn(__fsub_rn(iso, s), __fadd_rn(__fsub_rn(s1, s), 1.0e-10f));
}

// 8 bits -> bit positions 0, 4, 8, ..., 28.
__device__ __forceinline__ uint32_t spread8(uint32_t x) {
  x &= 0xffu;
  x = (x | (x << 12)) & 0x000f000fu;
  x = (x | (x << 6)) & 0x03030303u;
  x = (x | (x << 3)) & 0x11111111u;
  return x;
}

// ------------------------------------------------------------------------
// decoupled look-back (single-pass scan across tiles)
// ------------------------------------------------------------------------
//
// Tile t publishes flags[t] = 1 with its aggregate, then flags[t] = 2 with
// its inclusive prefix.  Called by all 32 lanes of one warp; every lane
// returns the exclusive prefix.  A wait longer than wait_ns (measured with
// %globaltimer) gives up, records TKMC_ERR_DEVICE_TIMEOUT in *err and
// publishes anyway so later tiles do not wait on this one.
template <int K>
__device__ void lookback(uint32_t* flags, long long* agg, long long* incl,
                         int64_t tile, const long long (&aggregate)[K],
                         long long (&prefix)[K], int64_t wait_ns,
                         bool skip_publish, long long* err) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < K; ++k) prefix[k] = 0;
  if (tile > 0 && lane == 0 && !skip_publish) {
#pragma unroll
    for (int k = 0; k < K; ++k) agg[tile * K + k] = aggregate[k];
    st_release_u32(flags + tile, 1u);
  }
  bool timed_out = false;
  if (tile > 0) {
    int64_t pred = tile - 1;
    uint64_t t0 = 0;
    while (true) {
      const int64_t idx = pred - lane;
      const uint32_t f = idx >= 0 ? ld_acquire_u32(flags + idx) : 2u;
      const uint32_t m2 = __ballot_sync(0xffffffffu, f == 2u);
      const uint32_t m0 = __ballot_sync(0xffffffffu, f == 0u);
      const uint32_t need = m2 ? (((m2 & (0u - m2)) << 1) - 1u) : 0xffffffffu;
      if (m0 & need) {
        uint64_t now = 0;
        if (lane == 0) now = global_ns();
        now = __shfl_sync(0xffffffffu, now, 0);
        if (t0 == 0) t0 = now;
        if ((int64_t)(now - t0) > wait_ns) {
          timed_out = true;
          break;
        }
        __nanosleep(64);
        continue;
      }
      const int first2 = m2 ? __ffs(m2) - 1 : 32;
      const bool take = ((need >> lane) & 1u) && idx >= 0;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        long long v = 0;
        if (take) v = (lane == first2) ? __ldcg(incl + idx * K + k) : __ldcg(agg + idx * K + k);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        prefix[k] += v;
      }
      if (m2) break;
      pred -= 32;
    }
  }
  if (lane == 0 && !skip_publish) {
#pragma unroll
    for (int k = 0; k < K; ++k) incl[tile * K + k] = prefix[k] + aggregate[k];
    st_release_u32(flags + tile, 2u);
  }
  if (timed_out && lane == 0) atomicExch((unsigned long long*)err, (unsigned long long)TKMC_ERR_DEVICE_TIMEOUT);
}

// ------------------------------------------------------------------------
// K1: threshold the volume into node bitmasks (all isovalues, one read)
// ------------------------------------------------------------------------
//
// A warp takes 1024 consecutive nodes (4 KiB) per step: eight coalesced
// 512-byte float4 loads, issued before any use.  Four ballots per load give
// the "above" bits in lane-interleaved order; each lane assembles one 32-bit
// word of node order and the warp stores 32 words (128 B) coalesced.
__global__ void __launch_bounds__(kThreads)
k_fe_threshold_v4(const float* __restrict__ v, int64_t n, IsoParams iso, int niso,
                  uint32_t* __restrict__ bits, int64_t bits_stride, int64_t nwords) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t nchunks = (n + 1023) >> 10;
  const float4* __restrict__ v4 = reinterpret_cast<const float4*>(v);
  if (blockIdx.x == 0 && threadIdx.x < 8 * TKMC_MAX_ISO) {
    const int t = threadIdx.x >> 3;
    if (t < niso) bits[t * bits_stride + nwords + (threadIdx.x & 7)] = 0u;  // padding
  }
  for (int64_t ch = warp; ch < nchunks; ch += nwarps) {
    const int64_t base = ch << 10;
    float4 x[8];
    if (base + 1024 <= n) {
#pragma unroll
      for (int q = 0; q < 8; ++q) x[q] = __ldcs(v4 + (base >> 2) + q * 32 + lane);
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int64_t e = base + q * 128 + lane * 4;
        x[q].x = e + 0 < n ? v[e + 0] : -INFINITY;
        x[q].y = e + 1 < n ? v[e + 1] : -INFINITY;
        x[q].z = e + 2 < n ? v[e + 2] : -INFINITY;
        x[q].w = e + 3 < n ? v[e + 3] : -INFINITY;
      }
    }
    const int64_t wi = (ch << 5) + lane;
    const int sh = (lane & 3) * 8;
    for (int t = 0; t < niso; ++t) {
      const float th = iso.v[t];
      uint32_t word = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t b0 = __ballot_sync(0xffffffffu, x[q].x > th);
        const uint32_t b1 = __ballot_sync(0xffffffffu, x[q].y > th);
        const uint32_t b2 = __ballot_sync(0xffffffffu, x[q].z > th);
        const uint32_t b3 = __ballot_sync(0xffffffffu, x[q].w > th);
        if ((lane >> 2) == q)
          word = spread8(b0 >> sh) | (spread8(b1 >> sh) << 1) |
                 (spread8(b2 >> sh) << 2) | (spread8(b3 >> sh) << 3);
      }
      if (wi < nwords) bits[t * bits_stride + wi] = word;
    }
  }
}

// Same result for a volume pointer that is not 16-byte aligned: 32 scalar
// coalesced loads per warp step, one ballot per word.
__global__ void __launch_bounds__(kThreads)
k_fe_threshold_scalar(const float* __restrict__ v, int64_t n, IsoParams iso, int niso,
                      uint32_t* __restrict__ bits, int64_t bits_stride, int64_t nwords) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t nchunks = (n + 1023) >> 10;
  if (blockIdx.x == 0 && threadIdx.x < 8 * TKMC_MAX_ISO) {
    const int t = threadIdx.x >> 3;
    if (t < niso) bits[t * bits_stride + nwords + (threadIdx.x & 7)] = 0u;
  }
  for (int64_t ch = warp; ch < nchunks; ch += nwarps) {
    const int64_t base = ch << 10;
    float x[32];
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      const int64_t e = base + q * 32 + lane;
      x[q] = e < n ? __ldcs(v + e) : -INFINITY;
    }
    const int64_t wi = (ch << 5) + lane;
    for (int t = 0; t < niso; ++t) {
      const float th = iso.v[t];
      uint32_t word = 0;
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const uint32_t b = __ballot_sync(0xffffffffu, x[q] > th);
        if (lane == q) word = b;
      }
      if (wi < nwords) bits[t * bits_stride + wi] = word;
    }
  }
}

// ------------------------------------------------------------------------
// shared geometry of the fe passes
// ------------------------------------------------------------------------

struct FeDims {
  int64_t L, M, N;      // nodes per row, rows per plane, planes (incl. ghost)
  int64_t R;            // node rows = M * N
  int64_t n_own_rows;   // rows this slab owns (R, or R - M with a ghost plane)
  int64_t nx, ny;       // cells per row, cell rows per plane (mask index)
  int64_t ntiles;       // K2 tiles
  int W;                // 32-bit words per row
  int S, logS;          // lanes per row (power of two <= 32)
};

// Per-isovalue workspace views.
struct FeIsoWs {
  uint32_t* bits;       // flat node bitmask
  long long* rowoff;    // [R][4] exclusive offsets X, Y, Z, T (section-relative)
  uint32_t* work;       // active own rows
  uint32_t* flags;      // [ntiles]
  long long* agg;       // [ntiles][4]
  long long* incl;      // [ntiles][4]
  long long* info;      // [16]: 0-3 own totals, 4-7 all-row totals, 8 active rows,
                        //       9 tile counter, 10 error
};

struct FeWsAll {
  FeIsoWs iso[TKMC_MAX_ISO];
};

// Bits of four node rows around one word: a = (j,k), b = (j+1,k),
// c = (j,k+1), d = (j+1,k+1), each with the next word's bit 0 available
// through the *n values.
struct Quad {
  uint32_t a, b, c, d, an, bn, cn, dn;
};

// Lanes sl of one S-lane row segment hold words w = w0 + sl.  Fills the next
// word of each row from the neighbouring lane, or loads it at the segment end.
__device__ __forceinline__ void load_quad(Quad& q, const uint32_t* __restrict__ bits,
                                          const FeDims& d, int64_t rowbit, int w, int sl,
                                          bool valid, bool hasY, bool hasZ) {
  const int64_t L = d.L;
  const int64_t plane = d.L * d.M;
  const bool hasC = hasY && hasZ;
  q.a = valid ? row_word(bits, rowbit, w, L) : 0u;
  q.b = hasY ? row_word(bits, rowbit + L, w, L) : 0u;
  q.c = hasZ ? row_word(bits, rowbit + plane, w, L) : 0u;
  q.d = hasC ? row_word(bits, rowbit + plane + L, w, L) : 0u;
  q.an = __shfl_down_sync(0xffffffffu, q.a, 1, d.S);
  q.bn = __shfl_down_sync(0xffffffffu, q.b, 1, d.S);
  q.cn = __shfl_down_sync(0xffffffffu, q.c, 1, d.S);
  q.dn = __shfl_down_sync(0xffffffffu, q.d, 1, d.S);
  if (sl == d.S - 1) {
    const bool more = (w + 1) < d.W;
    q.an = (valid && more) ? row_word(bits, rowbit, w + 1, L) : 0u;
    q.bn = (hasY && more) ? row_word(bits, rowbit + L, w + 1, L) : 0u;
    q.cn = (hasZ && more) ? row_word(bits, rowbit + plane, w + 1, L) : 0u;
    q.dn = (hasC && more) ? row_word(bits, rowbit + plane + L, w + 1, L) : 0u;
  }
}

// Case index of the cell at bit `b` (corner order of flying_edges.py:463-471).
__device__ __forceinline__ int cell_case(int b, uint32_t a, uint32_t a1, uint32_t bb,
                                         uint32_t b1, uint32_t c, uint32_t c1,
                                         uint32_t dd, uint32_t d1) {
  return (int)(((a >> b) & 1u) | (((a1 >> b) & 1u) << 1) | (((b1 >> b) & 1u) << 2) |
               (((bb >> b) & 1u) << 3) | (((c >> b) & 1u) << 4) | (((c1 >> b) & 1u) << 5) |
               (((d1 >> b) & 1u) << 6) | (((dd >> b) & 1u) << 7));
}

// Cells of word w whose 8 corners are not all on one side.
__device__ __forceinline__ uint32_t active_cells(const Quad& q, uint32_t xcell_mask) {
  const uint32_t u = (q.a ^ q.b) | (q.a ^ q.c) | (q.a ^ q.d);
  const uint32_t un = (q.an ^ q.bn) | (q.an ^ q.cn) | (q.an ^ q.dn);
  return (u | shr1(u, un) | (q.a ^ shr1(q.a, q.an))) & xcell_mask;
}

// ------------------------------------------------------------------------
// K2: per-row counts + single-pass scan + worklist
// ------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads)
k_fe_count_scan(FeDims d, FeWsAll ws, const int32_t* __restrict__ mask, int64_t wait_ns,
                int64_t skip_tile) {
  __shared__ int s_cnt[4][kRowsPerTile];
  __shared__ int s_ntri[256];
  __shared__ long long s_wtot[4][kThreads / 32];
  __shared__ long long s_prefix[4];
  __shared__ int64_t s_tile;
  __shared__ unsigned s_wbase[kThreads / 32];

  const FeIsoWs& W = ws.iso[blockIdx.y];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  s_ntri[tid] = (int)(c_case_tris[tid] >> 60);
  if (tid == 0) s_tile = (int64_t)atomicAdd((unsigned long long*)(W.info + 9), 1ull);
  __syncthreads();
  const int64_t tile = s_tile;
  const int64_t row0 = tile * kRowsPerTile;
  const int S = d.S, G = 32 >> d.logS;
  const int seg = lane >> d.logS, sl = lane & (S - 1);

  for (int p = 0; p < S; ++p) {
    const int local = ((p << 3) + warp) * G + seg;
    const int64_t r = row0 + local;
    const bool valid = r < d.R;
    const int64_t j = valid ? r % d.M : 0, k = valid ? r / d.M : 0;
    const bool hasY = valid && (j + 1 < d.M);
    const bool hasZ = valid && (k + 1 < d.N);
    const bool hasC = hasY && hasZ;
    const int64_t rowbit = r * d.L;
    unsigned cX = 0, cY = 0, cZ = 0, cT = 0;
    for (int w0 = 0; w0 < d.W; w0 += S) {
      const int w = w0 + sl;
      Quad q;
      load_quad(q, W.bits, d, rowbit, w, sl, valid, hasY, hasZ);
      const uint32_t xm = low_mask((int)(d.L - 1 - 32 * (int64_t)w));
      cX += __popc((q.a ^ shr1(q.a, q.an)) & xm);
      if (hasY) cY += __popc(q.a ^ q.b);
      if (hasZ) cZ += __popc(q.a ^ q.c);
      if (hasC) {
        uint32_t act = active_cells(q, xm);
        if (act) {
          const uint32_t a1 = shr1(q.a, q.an), b1 = shr1(q.b, q.bn);
          const uint32_t c1 = shr1(q.c, q.cn), d1 = shr1(q.d, q.dn);
          while (act) {
            const int b = __ffs(act) - 1;
            act &= act - 1;
            int nt = s_ntri[cell_case(b, q.a, a1, q.b, b1, q.c, c1, q.d, d1)];
            if (nt && mask) {
              const int64_t cell = (k * d.ny + j) * d.nx + 32 * (int64_t)w + b;
              if (__ldg(mask + cell) != 0) nt = 0;
            }
            cT += nt;
          }
        }
      }
    }
    for (int o = S >> 1; o > 0; o >>= 1) {
      cX += __shfl_xor_sync(0xffffffffu, cX, o);
      cY += __shfl_xor_sync(0xffffffffu, cY, o);
      cZ += __shfl_xor_sync(0xffffffffu, cZ, o);
      cT += __shfl_xor_sync(0xffffffffu, cT, o);
    }
    if (sl == 0) {
      s_cnt[0][local] = (int)cX;
      s_cnt[1][local] = (int)cY;
      s_cnt[2][local] = (int)cZ;
      s_cnt[3][local] = (int)cT;
    }
  }
  __syncthreads();

  // Block-wide exclusive scan of the tile's 256 rows (thread tid <-> row tid).
  long long own[4], inc[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    own[c] = s_cnt[c][tid];
    long long x = own[c];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    inc[c] = x;
    if (lane == 31) s_wtot[c][warp] = x;
  }
  __syncthreads();
  long long tile_total[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    long long before = 0, all = 0;
#pragma unroll
    for (int w2 = 0; w2 < kThreads / 32; ++w2) {
      const long long t = s_wtot[c][w2];
      if (w2 < warp) before += t;
      all += t;
    }
    inc[c] += before;
    tile_total[c] = all;
  }
  if (warp == 0) {
    long long pre[4];
    lookback<4>(W.flags, W.agg, W.incl, tile, tile_total, pre, wait_ns,
                tile == skip_tile, W.info + 10);
    if (lane == 0)
#pragma unroll
      for (int c = 0; c < 4; ++c) s_prefix[c] = pre[c];
  }
  __syncthreads();

  const int64_t r = row0 + tid;
  long long ex[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) ex[c] = s_prefix[c] + inc[c] - own[c];
  if (r < d.R) {
    longlong2* dst = reinterpret_cast<longlong2*>(W.rowoff + r * 4);
    dst[0] = make_longlong2(ex[0], ex[1]);
    dst[1] = make_longlong2(ex[2], ex[3]);
    if (r == d.n_own_rows)
#pragma unroll
      for (int c = 0; c < 4; ++c) W.info[c] = ex[c];
    if (r == d.R - 1) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        W.info[4 + c] = ex[c] + own[c];
        if (d.n_own_rows == d.R) W.info[c] = ex[c] + own[c];
      }
    }
  }
  // Worklist of own rows with any output (order is irrelevant: every row
  // writes at its own offsets).
  const bool active = r < d.n_own_rows && (own[0] | own[1] | own[2] | own[3]) != 0;
  const uint32_t bal = __ballot_sync(0xffffffffu, active);
  if (lane == 0 && bal)
    s_wbase[warp] = (unsigned)atomicAdd((unsigned long long*)(W.info + 8),
                                        (unsigned long long)__popc(bal));
  __syncwarp();
  if (active) W.work[s_wbase[warp] + __popc(bal & ((1u << lane) - 1u))] = (uint32_t)r;
}

// ------------------------------------------------------------------------
// K3: emit points and triangles of the active rows
// ------------------------------------------------------------------------

struct FeEmitArgs {
  const float* v;
  const int32_t* mask;
  float* points;
  int32_t* conn;
  float geom[6];
  int64_t k_offset;
  IsoParams iso;
  long long pt_id_base[TKMC_MAX_ISO][3];
  long long pt_out_base[TKMC_MAX_ISO][3];
  long long tri_out_base[TKMC_MAX_ISO];
};

// Segmented (width S) inclusive scan.
__device__ __forceinline__ unsigned seg_scan(unsigned x, int sl, int S) {
  for (int o = 1; o < S; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, x, o, S);
    if (sl >= o) x += y;
  }
  return x;
}

__global__ void __launch_bounds__(kThreads)
k_fe_emit(FeDims d, FeWsAll ws, FeEmitArgs A) {
  __shared__ uint64_t s_case[256];
  __shared__ int s_pid[12][kThreads];
  const int isoi = blockIdx.y;
  const FeIsoWs& W = ws.iso[isoi];
  const int tid = threadIdx.x, lane = tid & 31;
  s_case[tid] = c_case_tris[tid];
  __syncthreads();

  const int S = d.S, G = 32 >> d.logS;
  const int seg = lane >> d.logS, sl = lane & (S - 1);
  const int64_t L = d.L, plane = d.L * d.M;
  const int64_t n_active = *((volatile long long*)(W.info + 8));
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + tid) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const float iso = A.iso.v[isoi];
  const float x0 = A.geom[0], y0 = A.geom[1], z0 = A.geom[2];
  const float hx = A.geom[3], hy = A.geom[4], hz = A.geom[5];
  const long long idX = A.pt_id_base[isoi][0], idY = A.pt_id_base[isoi][1],
                  idZ = A.pt_id_base[isoi][2];
  const long long outX = A.pt_out_base[isoi][0], outY = A.pt_out_base[isoi][1],
                  outZ = A.pt_out_base[isoi][2];
  const long long outT = A.tri_out_base[isoi];

  for (int64_t grp = gw; grp * G < n_active; grp += nw) {
    const int64_t item = grp * G + seg;
    const bool valid = item < n_active;
    const int64_t r = valid ? (int64_t)W.work[item] : 0;
    const int64_t j = r % d.M, k = r / d.M;
    const bool hasY = valid && (j + 1 < d.M);
    const bool hasZ = valid && (k + 1 < d.N);
    const bool hasC = hasY && hasZ;
    const int64_t rowbit = r * L;
    // Row offsets (section-relative) of the four node rows and the cell row.
    long long oxa = 0, oya = 0, oza = 0, ota = 0, oxb = 0, ozb = 0, oxc = 0, oyc = 0, oxd = 0;
    if (valid) {
      const longlong2* ra = reinterpret_cast<const longlong2*>(W.rowoff + r * 4);
      const longlong2 p0 = ra[0], p1 = ra[1];
      oxa = p0.x; oya = p0.y; oza = p1.x; ota = p1.y;
    }
    if (hasY) { oxb = W.rowoff[(r + 1) * 4 + 0]; ozb = W.rowoff[(r + 1) * 4 + 2]; }
    if (hasZ) { oxc = W.rowoff[(r + d.M) * 4 + 0]; oyc = W.rowoff[(r + d.M) * 4 + 1]; }
    if (hasC) oxd = W.rowoff[(r + d.M + 1) * 4 + 0];
    const float py = coord(y0, j, hy);
    const float pz = coord(z0, k + A.k_offset, hz);
    const float py1 = coord(y0, j + 1, hy);
    const float pz1 = coord(z0, k + 1 + A.k_offset, hz);

    unsigned cxa = 0, cya = 0, cza = 0, cxb = 0, cxc = 0, cxd = 0, cyc = 0, czb = 0, ct = 0;
    for (int w0 = 0; w0 < d.W; w0 += S) {
      const int w = w0 + sl;
      Quad q;
      load_quad(q, W.bits, d, rowbit, w, sl, valid, hasY, hasZ);
      const uint32_t xm = low_mask((int)(L - 1 - 32 * (int64_t)w));
      const uint32_t xa = (q.a ^ shr1(q.a, q.an)) & xm;
      const uint32_t ya = hasY ? (q.a ^ q.b) : 0u;
      const uint32_t za = hasZ ? (q.a ^ q.c) : 0u;
      uint32_t xb = 0, xc = 0, xd = 0, yc = 0, zb = 0, act = 0;
      uint32_t a1 = 0, b1 = 0, c1 = 0, d1 = 0;
      unsigned nt_lane = 0;
      if (hasC) {
        a1 = shr1(q.a, q.an); b1 = shr1(q.b, q.bn);
        c1 = shr1(q.c, q.cn); d1 = shr1(q.d, q.dn);
        xb = (q.b ^ b1) & xm;
        xc = (q.c ^ c1) & xm;
        xd = (q.d ^ d1) & xm;
        yc = q.c ^ q.d;
        zb = q.b ^ q.d;
        act = active_cells(q, xm);
        uint32_t m = act;
        while (m) {
          const int b = __ffs(m) - 1;
          m &= m - 1;
          unsigned nt = (unsigned)(s_case[cell_case(b, q.a, a1, q.b, b1, q.c, c1, q.d, d1)] >> 60);
          if (nt && A.mask) {
            const int64_t cell = (k * d.ny + j) * d.nx + 32 * (int64_t)w + b;
            if (__ldg(A.mask + cell) != 0) nt = 0;
          }
          if (!nt) act &= ~(1u << b);
          nt_lane += nt;
        }
      }
      // Segmented scans of the per-word counts, two 16-bit counts per lane.
      const unsigned p0 = __popc(xa) | (__popc(ya) << 16);
      const unsigned p1 = __popc(za) | (__popc(xb) << 16);
      const unsigned p2 = __popc(xc) | (__popc(xd) << 16);
      const unsigned p3 = __popc(yc) | (__popc(zb) << 16);
      const unsigned i0 = seg_scan(p0, sl, S), i1 = seg_scan(p1, sl, S);
      const unsigned i2 = seg_scan(p2, sl, S), i3 = seg_scan(p3, sl, S);
      const unsigned i4 = seg_scan(nt_lane, sl, S);
      const unsigned e0 = i0 - p0, e1 = i1 - p1, e2 = i2 - p2, e3 = i3 - p3, e4 = i4 - nt_lane;

      const int64_t nbase = rowbit;  // node index of (0, j, k)
      // ---- points of this node row: x, y, z sections ----
      {
        long long rel = oxa + cxa + (e0 & 0xffffu);
        uint32_t m = xa;
        while (m) {
          const int b = __ffs(m) - 1;
          m &= m - 1;
          const int64_t i = 32 * (int64_t)w + b;
          const float s = __ldg(A.v + nbase + i), s1 = __ldg(A.v + nbase + i + 1);
          const float t = interp_t(iso, s, s1);
          const float px = coord(x0, i, hx), px1 = coord(x0, i + 1, hx);
          float* o = A.points + (outX + rel) * 3;
          o[0] = lerp_ref(px, px1, t);
          o[1] = lerp_ref(py, py, t);
          o[2] = lerp_ref(pz, pz, t);
          ++rel;
        }
      }
      {
        long long rel = oya + cya + (e0 >> 16);
        uint32_t m = ya;
        while (m) {
          const int b = __ffs(m) - 1;
          m &= m - 1;
          const int64_t i = 32 * (int64_t)w + b;
          const float s = __ldg(A.v + nbase + i), s1 = __ldg(A.v + nbase + L + i);
          const float t = interp_t(iso, s, s1);
          const float px = coord(x0, i, hx);
          float* o = A.points + (outY + rel) * 3;
          o[0] = lerp_ref(px, px, t);
          o[1] = lerp_ref(py, py1, t);
          o[2] = lerp_ref(pz, pz, t);
          ++rel;
        }
      }
      {
        long long rel = oza + cza + (e1 & 0xffffu);
        uint32_t m = za;
        while (m) {
          const int b = __ffs(m) - 1;
          m &= m - 1;
          const int64_t i = 32 * (int64_t)w + b;
          const float s = __ldg(A.v + nbase + i), s1 = __ldg(A.v + nbase + plane + i);
          const float t = interp_t(iso, s, s1);
          const float px = coord(x0, i, hx);
          float* o = A.points + (outZ + rel) * 3;
          o[0] = lerp_ref(px, px, t);
          o[1] = lerp_ref(py, py, t);
          o[2] = lerp_ref(pz, pz1, t);
          ++rel;
        }
      }
      // ---- triangles of this cell row ----
      if (act) {
        const long long Pxa = idX + oxa + cxa + (e0 & 0xffffu);
        const long long Pya = idY + oya + cya + (e0 >> 16);
        const long long Pza = idZ + oza + cza + (e1 & 0xffffu);
        const long long Pxb = idX + oxb + cxb + (e1 >> 16);
        const long long Pxc = idX + oxc + cxc + (e2 & 0xffffu);
        const long long Pxd = idX + oxd + cxd + (e2 >> 16);
        const long long Pyc = idY + oyc + cyc + (e3 & 0xffffu);
        const long long Pzb = idZ + ozb + czb + (e3 >> 16);
        long long tpos = outT + ota + ct + e4;
        uint32_t m = act;
        while (m) {
          const int b = __ffs(m) - 1;
          m &= m - 1;
          const uint32_t lo = low_mask(b), lo1 = low_mask(b + 1);
          s_pid[0][tid] = (int)(Pxa + __popc(xa & lo));
          s_pid[1][tid] = (int)(Pya + __popc(ya & lo1));
          s_pid[2][tid] = (int)(Pxb + __popc(xb & lo));
          s_pid[3][tid] = (int)(Pya + __popc(ya & lo));
          s_pid[4][tid] = (int)(Pxc + __popc(xc & lo));
          s_pid[5][tid] = (int)(Pyc + __popc(yc & lo1));
          s_pid[6][tid] = (int)(Pxd + __popc(xd & lo));
          s_pid[7][tid] = (int)(Pyc + __popc(yc & lo));
          s_pid[8][tid] = (int)(Pza + __popc(za & lo));
          s_pid[9][tid] = (int)(Pza + __popc(za & lo1));
          s_pid[10][tid] = (int)(Pzb + __popc(zb & lo));
          s_pid[11][tid] = (int)(Pzb + __popc(zb & lo1));
          const uint64_t pk = s_case[cell_case(b, q.a, a1, q.b, b1, q.c, c1, q.d, d1)];
          const int nt = (int)(pk >> 60);
          int32_t* o = A.conn + tpos * 3;
          for (int t = 0; t < 3 * nt; ++t) o[t] = s_pid[(pk >> (4 * t)) & 0xfu][tid];
          tpos += nt;
        }
      }
      // Carry the segment totals to the next chunk of words.
      const unsigned t0 = __shfl_sync(0xffffffffu, i0, S - 1, S);
      const unsigned t1 = __shfl_sync(0xffffffffu, i1, S - 1, S);
      const unsigned t2 = __shfl_sync(0xffffffffu, i2, S - 1, S);
      const unsigned t3 = __shfl_sync(0xffffffffu, i3, S - 1, S);
      const unsigned t4 = __shfl_sync(0xffffffffu, i4, S - 1, S);
      cxa += t0 & 0xffffu; cya += t0 >> 16;
      cza += t1 & 0xffffu; cxb += t1 >> 16;
      cxc += t2 & 0xffffu; cxd += t2 >> 16;
      cyc += t3 & 0xffffu; czb += t3 >> 16;
      ct += t4;
    }
  }
}

// ------------------------------------------------------------------------
// per-cell classification (26_marching_cubes.py:435-450)
// ------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads)
k_mc_classify_cells(const uint32_t* __restrict__ bits, int64_t L, int64_t M, int64_t nx,
                    int64_t ny, int64_t ncells, const int32_t* __restrict__ mask,
                    uint8_t* __restrict__ cases, int32_t* __restrict__ ntris) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < ncells; c += stride) {
    const int64_t i = c % nx, j = (c / nx) % ny, k = c / (nx * ny);
    const int64_t n0 = (k * M + j) * L + i;
    auto bit = [&](int64_t n) -> int { return (int)((__ldg(bits + (n >> 5)) >> (n & 31)) & 1u); };
    const int64_t P = L * M;
    const int cs = bit(n0) | (bit(n0 + 1) << 1) | (bit(n0 + L + 1) << 2) | (bit(n0 + L) << 3) |
                   (bit(n0 + P) << 4) | (bit(n0 + P + 1) << 5) | (bit(n0 + P + L + 1) << 6) |
                   (bit(n0 + P + L) << 7);
    if (cases) cases[c] = (uint8_t)cs;
    if (ntris) ntris[c] = (mask && mask[c] != 0) ? 0 : (int32_t)(c_case_tris[cs] >> 60);
  }
}

// ------------------------------------------------------------------------
// field reduction: min / max (NaN ignored), sum (f64), NaN count
// ------------------------------------------------------------------------

struct RedPart {
  float mn, mx;
  double sum;
  long long nan;
};

__device__ __forceinline__ void red_add(RedPart& p, float x) {
  if (x != x) {
    ++p.nan;
  } else {
    p.mn = fminf(p.mn, x);
    p.mx = fmaxf(p.mx, x);
  }
  p.sum += (double)x;
}

__device__ __forceinline__ void red_merge(RedPart& p, const RedPart& q) {
  p.mn = fminf(p.mn, q.mn);
  p.mx = fmaxf(p.mx, q.mx);
  p.sum += q.sum;
  p.nan += q.nan;
}

__device__ RedPart red_block(RedPart p) {
  __shared__ RedPart s_part[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    RedPart q;
    q.mn = __shfl_xor_sync(0xffffffffu, p.mn, o);
    q.mx = __shfl_xor_sync(0xffffffffu, p.mx, o);
    q.sum = __shfl_xor_sync(0xffffffffu, p.sum, o);
    q.nan = __shfl_xor_sync(0xffffffffu, p.nan, o);
    red_merge(p, q);
  }
  if (lane == 0) s_part[warp] = p;
  __syncthreads();
  RedPart r = s_part[0];
  for (int w = 1; w < kThreads / 32; ++w) red_merge(r, s_part[w]);
  return r;
}

__global__ void __launch_bounds__(kThreads)
k_reduce_partial(const float* __restrict__ v, int64_t n, int vec, RedPart* __restrict__ parts) {
  RedPart p{INFINITY, -INFINITY, 0.0, 0};
  const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t done = 0;
  if (vec) {
    const float4* v4 = reinterpret_cast<const float4*>(v);
    const int64_t n4 = n >> 2;
    for (int64_t i = gt; i < n4; i += stride) {
      const float4 x = __ldcs(v4 + i);
      red_add(p, x.x); red_add(p, x.y); red_add(p, x.z); red_add(p, x.w);
    }
    done = n4 << 2;
  }
  for (int64_t i = done + gt; i < n; i += stride) red_add(p, __ldcs(v + i));
  const RedPart r = red_block(p);
  if (threadIdx.x == 0) parts[blockIdx.x] = r;
}

__global__ void __launch_bounds__(kThreads)
k_reduce_final(const RedPart* __restrict__ parts, int nparts, double* __restrict__ out4) {
  RedPart p{INFINITY, -INFINITY, 0.0, 0};
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) red_merge(p, parts[i]);
  const RedPart r = red_block(p);
  if (threadIdx.x == 0) {
    out4[0] = (double)r.mn;
    out4[1] = (double)r.mx;
    out4[2] = r.sum;
    out4[3] = (double)r.nan;
  }
}

// ------------------------------------------------------------------------
// generic int32 scan (decoupled look-back)
// ------------------------------------------------------------------------
// Each warp scans 512 consecutive items as 16 coalesced rounds of 32 with a
// running carry; warps combine through shared memory; tiles through the
// look-back.  Int32 running sums wrap exactly as int64 sums truncated.
__global__ void __launch_bounds__(kThreads)
k_scan_i32(const int32_t* in, int32_t* out, int64_t n, int inclusive, uint32_t* flags,
           long long* agg, long long* incl, long long* info, int64_t wait_ns, int64_t skip_tile) {
  __shared__ long long s_wtot[kThreads / 32];
  __shared__ long long s_prefix;
  __shared__ int64_t s_tile;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_tile = (int64_t)atomicAdd((unsigned long long*)(info + 0), 1ull);
  __syncthreads();
  const int64_t tile = s_tile;
  const int64_t base = tile * kScanTile + (int64_t)warp * (32 * kScanItems);
  int32_t x[kScanItems], ex[kScanItems];
  int32_t carry = 0;
  long long wsum = 0;
#pragma unroll
  for (int q = 0; q < kScanItems; ++q) {
    const int64_t e = base + q * 32 + lane;
    x[q] = e < n ? in[e] : 0;
    int32_t s = x[q];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s = (int32_t)((uint32_t)s + (uint32_t)y);
    }
    ex[q] = (int32_t)((uint32_t)carry + (uint32_t)s - (uint32_t)x[q]);
    carry = (int32_t)((uint32_t)carry + (uint32_t)__shfl_sync(0xffffffffu, s, 31));
    long long v = x[q];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    wsum += v;
  }
  if (lane == 0) s_wtot[warp] = wsum;
  __syncthreads();
  long long before = 0, total = 0;
  for (int w = 0; w < kThreads / 32; ++w) {
    if (w < warp) before += s_wtot[w];
    total += s_wtot[w];
  }
  if (warp == 0) {
    long long agg1[1] = {total}, pre[1];
    lookback<1>(flags, agg, incl, tile, agg1, pre, wait_ns, tile == skip_tile, info + 2);
    if (lane == 0) s_prefix = pre[0];
  }
  __syncthreads();
  const uint32_t off = (uint32_t)(unsigned long long)(s_prefix + before);
#pragma unroll
  for (int q = 0; q < kScanItems; ++q) {
    const int64_t e = base + q * 32 + lane;
    if (e < n) out[e] = (int32_t)(off + (uint32_t)ex[q] + (inclusive ? (uint32_t)x[q] : 0u));
  }
  if (tid == 0 && (tile + 1) * kScanTile >= n) info[1] = s_prefix + total;
}

// ------------------------------------------------------------------------
// host: fe workspace layout
// ------------------------------------------------------------------------

struct FeLayout {
  FeDims d;
  int64_t V, nwords, bits_stride;
  size_t off_bits, off_rowoff, off_work, off_info, off_flags, off_agg, off_incl, total;
  size_t reset_bytes;  // info + flags, zeroed before each scan
};

bool fe_layout(int64_t nx, int64_t ny, int64_t nz, int ghost, int niso, FeLayout* out) {
  if (nx < 0 || ny < 0 || nz < 0 || niso < 1 || niso > TKMC_MAX_ISO) return false;
  if (ghost && nz < 1) return false;
  FeLayout f{};
  FeDims& d = f.d;
  d.L = nx + 1;
  d.M = ny + 1;
  d.N = nz + 1;
  d.R = d.M * d.N;
  d.n_own_rows = ghost ? d.R - d.M : d.R;
  d.nx = nx;
  d.ny = ny;
  const int64_t W = (d.L + 31) / 32;
  if (W > (1 << 24)) return false;
  d.W = (int)W;
  int S = 1, logS = 0;
  while (S < d.W && S < 32) { S <<= 1; ++logS; }
  d.S = S;
  d.logS = logS;
  d.ntiles = (d.R + kRowsPerTile - 1) / kRowsPerTile;
  if (d.R > 0xffffffffLL) return false;  // worklist holds uint32 row ids
  f.V = d.L * d.M * d.N;
  f.nwords = (f.V + 31) / 32;
  f.bits_stride = (int64_t)align_up((size_t)(f.nwords + 8), 64);
  size_t o = 0;
  f.off_info = o;   o = align_up(o + (size_t)niso * 16 * 8, 256);
  f.off_flags = o;  o = align_up(o + (size_t)niso * d.ntiles * 4, 256);
  f.reset_bytes = o;
  f.off_agg = o;    o = align_up(o + (size_t)niso * d.ntiles * 4 * 8, 256);
  f.off_incl = o;   o = align_up(o + (size_t)niso * d.ntiles * 4 * 8, 256);
  f.off_rowoff = o; o = align_up(o + (size_t)niso * d.R * 4 * 8, 256);
  f.off_work = o;   o = align_up(o + (size_t)niso * d.R * 4, 256);
  f.off_bits = o;   o = align_up(o + (size_t)niso * f.bits_stride * 4, 256);
  f.total = o;
  *out = f;
  return true;
}

FeWsAll fe_views(const FeLayout& f, void* ws, int niso) {
  FeWsAll a{};
  char* b = static_cast<char*>(ws);
  for (int q = 0; q < niso; ++q) {
    FeIsoWs& w = a.iso[q];
    w.bits = reinterpret_cast<uint32_t*>(b + f.off_bits) + (size_t)q * f.bits_stride;
    w.rowoff = reinterpret_cast<long long*>(b + f.off_rowoff) + (size_t)q * f.d.R * 4;
    w.work = reinterpret_cast<uint32_t*>(b + f.off_work) + (size_t)q * f.d.R;
    w.flags = reinterpret_cast<uint32_t*>(b + f.off_flags) + (size_t)q * f.d.ntiles;
    w.agg = reinterpret_cast<long long*>(b + f.off_agg) + (size_t)q * f.d.ntiles * 4;
    w.incl = reinterpret_cast<long long*>(b + f.off_incl) + (size_t)q * f.d.ntiles * 4;
    w.info = reinterpret_cast<long long*>(b + f.off_info) + (size_t)q * 16;
  }
  return a;
}

int check_ws(void* ws, size_t have, size_t need) {
  if (need && !ws) return set_err(TKMC_ERR_INVALID_ARG, "workspace is NULL");
  if (have < need)
    return set_err(TKMC_ERR_WORKSPACE, "workspace too small: %zu bytes given, %zu needed", have,
                   need);
  if (reinterpret_cast<uintptr_t>(ws) % 256)
    return set_err(TKMC_ERR_INVALID_ARG, "workspace must be 256-byte aligned");
  return TKMC_OK;
}

int check_iso(const float* isovalues, int niso) {
  if (!isovalues) return set_err(TKMC_ERR_INVALID_ARG, "isovalues is NULL");
  if (niso < 1 || niso > TKMC_MAX_ISO)
    return set_err(TKMC_ERR_INVALID_ARG, "niso must be in [1, %d], got %d", TKMC_MAX_ISO, niso);
  return TKMC_OK;
}

int grid_for(int64_t work_items, int per_block, int blocks_per_sm) {
  int64_t g = (work_items + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * blocks_per_sm;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

}  // namespace

// ==========================================================================
// C ABI
// ==========================================================================

extern "C" {

int tkmc_version(void) { return TKMC_VERSION; }

const char* tkmc_last_error(void) { return g_err; }

uint64_t tkmc_launch_count(void) { return g_launches.load(); }

void tkmc_set_wait_limit_ns(int64_t ns) { g_wait_ns.store(ns > 0 ? ns : 1000000000LL); }

void tkmc_test_skip_publish(int64_t tile) { g_skip_tile.store(tile); }

int tkmc_mc_tables(int32_t* tri_table, int32_t* num_tris, int32_t* edge_corners) {
  tkmc::unpack_tri_table(tri_table, num_tris);
  if (edge_corners)
    for (int i = 0; i < 24; ++i) edge_corners[i] = tkmc::kEdgeCorners[i];
  return TKMC_OK;
}

// ---- reductions ----------------------------------------------------------

static int reduce_grid(int64_t n) { return grid_for((n + 3) / 4, kThreads * 8, 4); }

size_t tkmc_reduce_workspace_bytes(int64_t n) {
  if (n < 0) return 0;
  return align_up((size_t)reduce_grid(n) * sizeof(RedPart), 256) + 256;
}

int tkmc_reduce_f32(const float* values, int64_t n, void* ws, size_t ws_bytes, double* out4,
                    void* stream) {
  if (n < 0 || !out4 || (n > 0 && !values))
    return set_err(TKMC_ERR_INVALID_ARG, "tkmc_reduce_f32: bad arguments");
  const size_t need = tkmc_reduce_workspace_bytes(n);
  int rc = check_ws(ws, ws_bytes, need);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int g = reduce_grid(n);
  RedPart* parts = static_cast<RedPart*>(ws);
  double* dout = reinterpret_cast<double*>(static_cast<char*>(ws) + need - 256);
  const int vec = (reinterpret_cast<uintptr_t>(values) % 16) == 0;
  k_reduce_partial<<<g, kThreads, 0, st>>>(values, n, vec, parts);
  TK_LAUNCHED();
  k_reduce_final<<<1, kThreads, 0, st>>>(parts, g, dout);
  TK_LAUNCHED();
  TK_CUDA(cudaMemcpyAsync(out4, dout, 4 * sizeof(double), cudaMemcpyDeviceToHost, st));
  TK_CUDA(cudaStreamSynchronize(st));
  return TKMC_OK;
}

// ---- scan ----------------------------------------------------------------

size_t tkmc_scan_workspace_bytes(int64_t n) {
  if (n < 0) return 0;
  const int64_t tiles = (n + kScanTile - 1) / kScanTile;
  return 256 + align_up((size_t)tiles * 4, 256) + 2 * align_up((size_t)tiles * 8, 256);
}

int tkmc_scan_i32(const int32_t* in, int32_t* out, int64_t n, int inclusive, void* ws,
                  size_t ws_bytes, int64_t* total, void* stream) {
  if (n < 0 || (n > 0 && (!in || !out)))
    return set_err(TKMC_ERR_INVALID_ARG, "tkmc_scan_i32: bad arguments");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    if (total) *total = 0;
    return TKMC_OK;
  }
  const size_t need = tkmc_scan_workspace_bytes(n);
  int rc = check_ws(ws, ws_bytes, need);
  if (rc) return rc;
  const int64_t tiles = (n + kScanTile - 1) / kScanTile;
  char* b = static_cast<char*>(ws);
  long long* info = reinterpret_cast<long long*>(b);  // 0 counter, 1 total, 2 error
  uint32_t* flags = reinterpret_cast<uint32_t*>(b + 256);
  long long* agg = reinterpret_cast<long long*>(b + 256 + align_up((size_t)tiles * 4, 256));
  long long* incl = agg + align_up((size_t)tiles * 8, 256) / 8;
  TK_CUDA(cudaMemsetAsync(ws, 0, 256 + align_up((size_t)tiles * 4, 256), st));
  const int64_t skip = g_skip_tile.exchange(-1);
  k_scan_i32<<<(unsigned)tiles, kThreads, 0, st>>>(in, out, n, inclusive, flags, agg, incl, info,
                                                   g_wait_ns.load(), skip);
  TK_LAUNCHED();
  if (total) {
    long long h[3];
    TK_CUDA(cudaMemcpyAsync(h, info, sizeof(h), cudaMemcpyDeviceToHost, st));
    TK_CUDA(cudaStreamSynchronize(st));
    if (h[2]) return set_err(TKMC_ERR_DEVICE_TIMEOUT, "scan look-back wait expired");
    *total = h[1];
  }
  return TKMC_OK;
}

// ---- flying edges --------------------------------------------------------

size_t tkmc_fe_workspace_bytes(int64_t nx, int64_t ny, int64_t nz, int niso) {
  FeLayout f;
  if (!fe_layout(nx, ny, nz, 0, niso, &f)) return 0;
  return f.total;
}

int tkmc_fe_classify(const float* scalar, int64_t nx, int64_t ny, int64_t nz,
                     const float* isovalues, int niso, void* ws, size_t ws_bytes, void* stream) {
  int rc = check_iso(isovalues, niso);
  if (rc) return rc;
  FeLayout f;
  if (!fe_layout(nx, ny, nz, 0, niso, &f))
    return set_err(TKMC_ERR_INVALID_ARG, "bad grid %lld x %lld x %lld", (long long)nx,
                   (long long)ny, (long long)nz);
  if (!scalar) return set_err(TKMC_ERR_INVALID_ARG, "scalar is NULL");
  if ((rc = check_ws(ws, ws_bytes, f.total))) return rc;
  IsoParams iso{};
  for (int t = 0; t < niso; ++t) iso.v[t] = isovalues[t];
  FeWsAll v = fe_views(f, ws, niso);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t nchunks = (f.V + 1023) / 1024;
  const int g = grid_for(nchunks, kThreads / 32, 8);
  uint32_t* bits0 = v.iso[0].bits;
  if ((reinterpret_cast<uintptr_t>(scalar) % 16) == 0)
    k_fe_threshold_v4<<<g, kThreads, 0, st>>>(scalar, f.V, iso, niso, bits0, f.bits_stride,
                                              f.nwords);
  else
    k_fe_threshold_scalar<<<g, kThreads, 0, st>>>(scalar, f.V, iso, niso, bits0, f.bits_stride,
                                                  f.nwords);
  TK_LAUNCHED();
  return TKMC_OK;
}

int tkmc_fe_scan(int64_t nx, int64_t ny, int64_t nz, int ghost_plane, int niso,
                 const int32_t* mask, void* ws, size_t ws_bytes, void* stream) {
  FeLayout f;
  if (!fe_layout(nx, ny, nz, ghost_plane, niso, &f))
    return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  int rc = check_ws(ws, ws_bytes, f.total);
  if (rc) return rc;
  FeWsAll v = fe_views(f, ws, niso);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  TK_CUDA(cudaMemsetAsync(static_cast<char*>(ws) + f.off_info, 0, f.reset_bytes - f.off_info, st));
  const int64_t skip = g_skip_tile.exchange(-1);
  dim3 grid((unsigned)f.d.ntiles, (unsigned)niso);
  k_fe_count_scan<<<grid, kThreads, 0, st>>>(f.d, v, mask, g_wait_ns.load(), skip);
  TK_LAUNCHED();
  return TKMC_OK;
}

int tkmc_fe_read_counts(int64_t nx, int64_t ny, int64_t nz, int niso, void* ws, size_t ws_bytes,
                        int64_t* counts, void* stream) {
  FeLayout f;
  if (!fe_layout(nx, ny, nz, 0, niso, &f)) return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  int rc = check_ws(ws, ws_bytes, f.total);
  if (rc) return rc;
  if (!counts) return set_err(TKMC_ERR_INVALID_ARG, "counts is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  long long h[TKMC_MAX_ISO * 16];
  TK_CUDA(cudaMemcpyAsync(h, static_cast<char*>(ws) + f.off_info, (size_t)niso * 16 * 8,
                          cudaMemcpyDeviceToHost, st));
  TK_CUDA(cudaStreamSynchronize(st));
  for (int q = 0; q < niso; ++q) {
    if (h[q * 16 + 10])
      return set_err(TKMC_ERR_DEVICE_TIMEOUT, "fe scan look-back wait expired (isovalue %d)", q);
    for (int c = 0; c < 4; ++c) counts[q * 4 + c] = h[q * 16 + c];
  }
  return TKMC_OK;
}

int tkmc_fe_row_offsets(int64_t nx, int64_t ny, int64_t nz, int niso, int iso,
                        const void* ws, size_t ws_bytes, int64_t* out, void* stream) {
  FeLayout f;
  if (!fe_layout(nx, ny, nz, 0, niso, &f)) return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  if (iso < 0 || iso >= niso) return set_err(TKMC_ERR_INVALID_ARG, "iso index out of range");
  int rc = check_ws(const_cast<void*>(ws), ws_bytes, f.total);
  if (rc) return rc;
  if (!out) return set_err(TKMC_ERR_INVALID_ARG, "out is NULL");
  FeWsAll v = fe_views(f, const_cast<void*>(ws), niso);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  TK_CUDA(cudaMemcpyAsync(out, v.iso[iso].rowoff, (size_t)f.d.R * 4 * sizeof(long long),
                          cudaMemcpyDeviceToHost, st));
  TK_CUDA(cudaStreamSynchronize(st));
  return TKMC_OK;
}

int tkmc_fe_count(const float* scalar, int64_t nx, int64_t ny, int64_t nz, int ghost_plane,
                  const float* isovalues, int niso, const int32_t* mask, void* ws,
                  size_t ws_bytes, int64_t* counts, void* stream) {
  int rc = tkmc_fe_classify(scalar, nx, ny, nz, isovalues, niso, ws, ws_bytes, stream);
  if (rc) return rc;
  if ((rc = tkmc_fe_scan(nx, ny, nz, ghost_plane, niso, mask, ws, ws_bytes, stream))) return rc;
  return tkmc_fe_read_counts(nx, ny, nz, niso, ws, ws_bytes, counts, stream);
}

int tkmc_fe_emit(const float* scalar, int64_t nx, int64_t ny, int64_t nz, int ghost_plane,
                 int64_t k_offset, const float* geom6, const float* isovalues, int niso,
                 const int32_t* mask, void* ws, size_t ws_bytes, const int64_t* pt_id_base,
                 const int64_t* pt_out_base, const int64_t* tri_out_base, float* points,
                 int32_t* conn, void* stream) {
  int rc = check_iso(isovalues, niso);
  if (rc) return rc;
  FeLayout f;
  if (!fe_layout(nx, ny, nz, ghost_plane, niso, &f))
    return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  if ((rc = check_ws(ws, ws_bytes, f.total))) return rc;
  if (!scalar || !geom6 || !pt_id_base || !pt_out_base || !tri_out_base)
    return set_err(TKMC_ERR_INVALID_ARG, "tkmc_fe_emit: NULL argument");
  FeEmitArgs A{};
  A.v = scalar;
  A.mask = mask;
  A.points = points;
  A.conn = conn;
  for (int i = 0; i < 6; ++i) A.geom[i] = geom6[i];
  A.k_offset = k_offset;
  for (int q = 0; q < niso; ++q) {
    A.iso.v[q] = isovalues[q];
    for (int s = 0; s < 3; ++s) {
      A.pt_id_base[q][s] = pt_id_base[3 * q + s];
      A.pt_out_base[q][s] = pt_out_base[3 * q + s];
    }
    A.tri_out_base[q] = tri_out_base[q];
  }
  FeWsAll v = fe_views(f, ws, niso);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int G = 32 >> f.d.logS;
  const int g = grid_for(f.d.n_own_rows, (kThreads / 32) * G, 8);
  dim3 grid((unsigned)g, (unsigned)niso);
  k_fe_emit<<<grid, kThreads, 0, st>>>(f.d, v, A);
  TK_LAUNCHED();
  return TKMC_OK;
}

int tkmc_fe_run(const float* scalar, int64_t nx, int64_t ny, int64_t nz, const float* geom6,
                const float* isovalues, int niso, const int32_t* mask, void* ws, size_t ws_bytes,
                float* points, int64_t points_capacity, int32_t* conn, int64_t conn_capacity,
                int64_t* counts, void* stream) {
  if (!counts) return set_err(TKMC_ERR_INVALID_ARG, "counts is NULL");
  int rc = tkmc_fe_count(scalar, nx, ny, nz, 0, isovalues, niso, mask, ws, ws_bytes, counts,
                         stream);
  if (rc) return rc;
  int64_t id[3 * TKMC_MAX_ISO], tri[TKMC_MAX_ISO];
  int64_t P = 0, T = 0;
  for (int q = 0; q < niso; ++q) {
    const int64_t X = counts[4 * q], Y = counts[4 * q + 1], Z = counts[4 * q + 2];
    id[3 * q] = P;
    id[3 * q + 1] = P + X;
    id[3 * q + 2] = P + X + Y;
    tri[q] = T;
    P += X + Y + Z;
    T += counts[4 * q + 3];
  }
  if (P > 0x7fffffffLL)
    return set_err(TKMC_ERR_OVERFLOW, "%lld points do not fit int32 point ids", (long long)P);
  if (P > points_capacity || T > conn_capacity)
    return set_err(TKMC_ERR_CAPACITY, "need %lld points / %lld triangles, capacity %lld / %lld",
                   (long long)P, (long long)T, (long long)points_capacity,
                   (long long)conn_capacity);
  if ((P > 0 && !points) || (T > 0 && !conn))
    return set_err(TKMC_ERR_INVALID_ARG, "output buffer is NULL");
  return tkmc_fe_emit(scalar, nx, ny, nz, 0, 0, geom6, isovalues, niso, mask, ws, ws_bytes, id,
                      id, tri, points, conn, stream);
}

int tkmc_mc_classify_cells(const float* scalar, int64_t nx, int64_t ny, int64_t nz,
                           float isovalue, const int32_t* mask, void* ws, size_t ws_bytes,
                           uint8_t* cases, int32_t* ntris, void* stream) {
  int rc = tkmc_fe_classify(scalar, nx, ny, nz, &isovalue, 1, ws, ws_bytes, stream);
  if (rc) return rc;
  FeLayout f;
  fe_layout(nx, ny, nz, 0, 1, &f);
  const int64_t ncells = nx * ny * nz;
  if (ncells == 0) return TKMC_OK;
  FeWsAll v = fe_views(f, ws, 1);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  k_mc_classify_cells<<<grid_for(ncells, kThreads, 8), kThreads, 0, st>>>(
      v.iso[0].bits, f.d.L, f.d.M, nx, ny, ncells, mask, cases, ntris);
  TK_LAUNCHED();
  return TKMC_OK;
}

}  // extern "C"
