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

// The eight edge groups around a cell row of word-granular emission: x(a)
// y(a) z(a) x(b) x(c) x(d) y(c) z(b), rows a = (j,k), b = (j+1,k),
// c = (j,k+1), d = (j+1,k+1).
// Edge e -> (group, +1 node) as nibble g | plus << 3 (edges 0..11).
constexpr uint64_t kEdgeGroup = 0x0ull | (0x9ull << 4) | (0x3ull << 8) | (0x1ull << 12) |
                                (0x4ull << 16) | (0xEull << 20) | (0x5ull << 24) |
                                (0x6ull << 28) | (0x2ull << 32) | (0xAull << 36) |
                                (0x7ull << 40) | (0xFull << 44);

constexpr uint64_t edge_group(int e) { return (kEdgeGroup >> (4 * e)) & 0xfull; }

// A case's triangle vertices as edge-group nibbles (g | plus << 3), nibble
// 15 the triangle count: the edge -> group step folded into the table.
constexpr uint64_t pack_case_groups(const char* s) {
  uint64_t w = 0;
  int n = 0;
  while (s[n]) {
    w |= edge_group(tkmc::hex_nibble(s[n])) << (4 * n);
    ++n;
  }
  return w | ((uint64_t)(n / 3) << 60);
}
#define TKMC_PACK_GROUPS(s) pack_case_groups(s),
__constant__ uint64_t c_case_groups[256] = {TKMC_CASE_LIST(TKMC_PACK_GROUPS)};
#undef TKMC_PACK_GROUPS

constexpr int kThreads = 256;
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

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization (launch_pdl) may start while the kernel before it in the
// stream is still running; griddep_wait() returns once that kernel has
// completed and its writes are visible, so it comes before the first read of
// anything the predecessor writes (it returns at once after a normal
// launch).  griddep_launch() lets the next such kernel launch as soon as
// every block of this grid has issued it.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

// p moved by off bytes.
template <typename T>
__device__ __forceinline__ T* shift_ptr(T* p, int64_t off) {
  return reinterpret_cast<T*>(reinterpret_cast<char*>(p) + off);
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

// ------------------------------------------------------------------------
// decoupled look-back (single-pass scan across tiles)
// ------------------------------------------------------------------------
//
// Tile t publishes flags[t] = 1 with its aggregate, then flags[t] = 2 with
// its inclusive prefix.  Called by all 32 lanes of one warp; every lane
// returns the exclusive prefix.  Each round inspects the 128 nearest
// unresolved predecessors (4 per lane): it sums aggregates back to the
// nearest inclusive prefix, or over all 128 and continues further back.  A
// wait longer than wait_ns (measured with %globaltimer) gives up, records
// TKMC_ERR_DEVICE_TIMEOUT in *err and publishes anyway so later tiles do
// not wait on this one.
template <int K>
__device__ void lookback(uint32_t* flags, long long* agg, long long* incl,
                         int64_t tile, const long long (&aggregate)[K],
                         long long (&prefix)[K], int64_t wait_ns,
                         bool skip_publish, long long* err) {
  constexpr int kPer = 4;  // predecessors per lane and round
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
      // Position p = kPer*lane + i is predecessor pred - p (p = 0 nearest).
      uint32_t f[kPer];
      int first2 = kPer, any0_before = 0;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int64_t idx = pred - (kPer * lane + i);
        f[i] = idx >= 0 ? ld_acquire_u32(flags + idx) : 2u;
      }
#pragma unroll
      for (int i = kPer - 1; i >= 0; --i)
        if (f[i] == 2u) first2 = i;
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        if (f[i] == 0u && i < first2) any0_before = 1;
      const uint32_t m2 = __ballot_sync(0xffffffffu, first2 < kPer);
      const int L2 = m2 ? __ffs(m2) - 1 : 32;  // lane holding the nearest inclusive
      // Not ready if a flag-0 predecessor is nearer than the nearest inclusive.
      const bool blocking = (lane < L2 && any0_before) ||
                            (lane == L2 && any0_before);
      if (__any_sync(0xffffffffu, blocking)) {
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
#pragma unroll
      for (int k = 0; k < K; ++k) {
        long long v = 0;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int64_t idx = pred - (kPer * lane + i);
          if (idx < 0) continue;
          if (lane < L2 || (lane == L2 && i < first2))
            v += __ldcg(agg + idx * K + k);
          else if (lane == L2 && i == first2)
            v += __ldcg(incl + idx * K + k);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        prefix[k] += v;
      }
      if (m2) break;
      pred -= 32 * kPer;
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
// A warp takes 1024 consecutive nodes (4 KiB): lane l loads nodes l, 32 + l,
// ..., 992 + l (32 coalesced 128-byte loads, all issued before any use), so
// each ballot over the warp is directly the bit word of 32 consecutive nodes
// and lane q keeps ballot q: per isovalue 32 compares, 32 ballots and 32
// selects, no interleave.  The warp stores its 32 words (128 B) coalesced.
// One chunk per warp and blocks in address order: the blocks in flight read
// one contiguous region of the volume.  (Eight float4 loads per lane with a
// four-way bit interleave after the ballots were 4-6 % slower for one
// isovalue and issue bound for several.)
//
// The same step leaves a summary of its 32 words: sums[ch] = {mixed, ones},
// bit w of `mixed` set when word 32*ch + w has nodes on both sides, bit w of
// `ones` when all its nodes are above.  The count pass reads these 8 bytes
// per 1024 nodes to find the few words where anything can change.

// Summary of the 32 words held by the warp's lanes (one word per lane).
__device__ __forceinline__ void store_summary(uint2* sums, int64_t ch, uint32_t word, int lane) {
  const uint32_t mixed = __ballot_sync(0xffffffffu, word != 0u && word != 0xffffffffu);
  const uint32_t ones = __ballot_sync(0xffffffffu, word == 0xffffffffu);
  if (lane == 0) sums[ch] = make_uint2(mixed, ones);
}

template <int NISO>
__device__ __forceinline__ void threshold_multi_body(const float* __restrict__ p, const IsoParams& iso,
                                                     uint32_t* __restrict__ bits, int64_t bits_stride,
                                                     uint2* __restrict__ sums, int64_t sums_stride,
                                                     int64_t ch, int lane) {
  float th[NISO];
  uint32_t word[NISO];
#pragma unroll
  for (int t = 0; t < NISO; ++t) {
    th[t] = iso.v[t];
    word[t] = 0u;
  }
  float x[32];
#pragma unroll
  for (int q = 0; q < 32; ++q) x[q] = __ldcs(p + 32 * q);
#pragma unroll
  for (int q = 0; q < 32; ++q) {
    const bool mine = lane == q;
#pragma unroll
    for (int t = 0; t < NISO; ++t) {
      const uint32_t b = __ballot_sync(0xffffffffu, x[q] > th[t]);
      word[t] = mine ? b : word[t];
    }
  }
  const int64_t wi = (ch << 5) + lane;
#pragma unroll
  for (int t = 0; t < NISO; ++t) {
    bits[t * bits_stride + wi] = word[t];
    store_summary(sums + t * sums_stride, ch, word[t], lane);
  }
}

// The isovalue count is a template parameter, so that the isovalues' ballot
// chains of one node column interleave (independent work for the scheduler)
// and share the lane test.  Several isovalues are issue bound: they run in
// 128-thread blocks at 12 per SM (48 warps), one isovalue in 256-thread
// blocks at 5 per SM.  Full chunks only; block 0 also zeroes the padding
// past the last word and the last summary.
template <int NISO>
constexpr int threshold_block() { return NISO == 1 ? 256 : 128; }

template <int NISO>
__global__ void __launch_bounds__(threshold_block<NISO>(), NISO == 1 ? 5 : 12)
k_fe_threshold_words(const float* __restrict__ v, int64_t nfull, IsoParams iso,
                     uint32_t* __restrict__ bits, int64_t bits_stride, int64_t nwords,
                     uint2* __restrict__ sums, int64_t sums_stride, int64_t nchunks,
                     int64_t ws_stride, const float* const* vols) {
  griddep_launch();
  // A batch of same-shape blocks: blockIdx.z picks the block.
  if (vols) v = vols[blockIdx.z];
  bits = shift_ptr(bits, (int64_t)blockIdx.z * ws_stride);
  sums = shift_ptr(sums, (int64_t)blockIdx.z * ws_stride);
  const int lane = threadIdx.x & 31;
  const int64_t ch = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (blockIdx.x == 0 && threadIdx.x < 8 * NISO) {
    const int t = threadIdx.x >> 3;
    bits[t * bits_stride + nwords + (threadIdx.x & 7)] = 0u;  // padding
    if ((threadIdx.x & 7) < 2)
      sums[t * sums_stride + nchunks + (threadIdx.x & 7)] = make_uint2(0u, 0u);
  }
  if (ch >= nfull) return;  // whole warps only
  threshold_multi_body<NISO>(v + (ch << 10) + lane, iso, bits, bits_stride, sums, sums_stride,
                             ch, lane);
}

// Launch K1 over nfull full chunks (blocks.z = nb same-shape volumes).
static void launch_threshold_words(int niso, int64_t nfull, unsigned nb, cudaStream_t st,
                                   const float* v, const IsoParams& iso, uint32_t* bits,
                                   int64_t bits_stride, int64_t nwords, uint2* sums,
                                   int64_t sums_stride, int64_t nchunks, int64_t ws_stride,
                                   const float* const* vols) {
#define TKMC_K1(N)                                                                            \
  case N: {                                                                                   \
    const int64_t per = threshold_block<N>() / 32;                                            \
    k_fe_threshold_words<N><<<dim3((unsigned)((nfull + per - 1) / per), 1, nb),                \
                              threshold_block<N>(), 0, st>>>(v, nfull, iso, bits, bits_stride, \
                                                             nwords, sums, sums_stride,        \
                                                             nchunks, ws_stride, vols);        \
    break;                                                                                    \
  }
  switch (niso) {  // 1 <= niso <= TKMC_MAX_ISO, checked by the callers
    TKMC_K1(1) TKMC_K1(2) TKMC_K1(3) TKMC_K1(4) TKMC_K1(5) TKMC_K1(6) TKMC_K1(7) TKMC_K1(8)
    default: break;
  }
#undef TKMC_K1
}

// Same result for a volume pointer that is not 16-byte aligned, and for the
// ragged last chunk of any volume: 32 scalar coalesced loads per warp step,
// one ballot per word.  Chunks first_chunk, first_chunk + 1, ... .
__global__ void __launch_bounds__(kThreads)
k_fe_threshold_scalar(const float* __restrict__ v, int64_t n, IsoParams iso, int niso,
                      uint32_t* __restrict__ bits, int64_t bits_stride, int64_t nwords,
                      uint2* __restrict__ sums, int64_t sums_stride, int64_t first_chunk,
                      int64_t ws_stride, const float* const* vols) {
  griddep_launch();
  // A batch of same-shape blocks: blockIdx.z picks the block.
  if (vols) v = vols[blockIdx.z];
  bits = shift_ptr(bits, (int64_t)blockIdx.z * ws_stride);
  sums = shift_ptr(sums, (int64_t)blockIdx.z * ws_stride);
  const int lane = threadIdx.x & 31;
  const int64_t warp = first_chunk + (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t nchunks = (n + 1023) >> 10;
  if (blockIdx.x == 0 && threadIdx.x < 8 * TKMC_MAX_ISO) {
    const int t = threadIdx.x >> 3;
    if (t < niso) bits[t * bits_stride + nwords + (threadIdx.x & 7)] = 0u;
    if (t < niso && (threadIdx.x & 7) < 2)
      sums[t * sums_stride + nchunks + (threadIdx.x & 7)] = make_uint2(0u, 0u);
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
      store_summary(sums + t * sums_stride, ch, word, lane);
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
  int64_t ntiles;       // scan tiles (K2b: kScanRows rows; aligned rows: kThreads rows)
  int64_t ctiles;       // K2a count tiles (rows not word-aligned)
  int W;                // 32-bit words per row
  int AW;               // words of the per-row activity mask = ceil(W / 32)
  int S, logS;          // lanes per row (power of two <= 32)
  int TR;               // K2 tile height in rows (rows not word-aligned)
  int logP;             // K2 threads per row = 1 << logP (TR << logP == block size)
  int S3, logS3;        // K3 lanes per row (<= 8: several rows per warp)
};

// One word of a node row with any output (word-aligned rows): the offsets,
// relative to their sections, of its first x, y and z point and of its
// first triangle.
struct FeUnit {
  uint32_t r, w;
  uint32_t xo, yo, zo, pad;
  long long to;
};

// Per-isovalue workspace views.
struct FeIsoWs {
  uint32_t* bits;       // flat node bitmask
  uint2* sums;          // per 32 words of bits: {mixed, ones} (see K1)
  int* cnt;             // [R][4] row counts X, Y, Z, T
  uint32_t* wact;       // [R][AW] words of each row with any output (bitmask)
  long long* tot;       // [4] this slab's own totals (contiguous across isovalues)
  long long* rowoff;    // [R][4] exclusive offsets X, Y, Z, T (section-relative)
  uint32_t* work;       // active own rows
  uint32_t* ufirst;     // [R] index of each row's first unit (word-aligned rows)
  uint32_t* ucnt;       // [R] units of each row (word-aligned rows)
  uint32_t* wcnt;       // [R][W] packed counts of each active word (word-aligned rows)
  FeUnit* units;        // units in (row, word) order, then a sentinel with the totals
  uint32_t* flags;      // [ntiles] (scan tiles of kScanRows rows)
  long long* super;     // [ntiles / kSuperTiles + 1][5] super-tile totals (word-aligned rows)
  long long* agg;       // [ntiles][4]
  long long* incl;      // [ntiles][4]
  long long* info;      // [16]: 0-3 own totals, 4-7 all-row totals, 8 active rows,
                        //       9 tile counter, 10 error, 11 units, 12 own units,
                        //       13 next emit task, 14 emit warps done
};

struct FeWsAll {
  FeIsoWs iso[TKMC_MAX_ISO];
  // A batch of blocks of one shape (blockIdx.z = block): their workspaces
  // `stride` bytes apart, and per block its volume, mask (entries may be
  // null) and geometry {x0, y0, z0, dx, dy, dz}.  stride = 0 and null
  // tables for one volume.
  int64_t stride;
  const float* const* vols;
  const int32_t* const* masks;
  const float* geoms;
};

// Workspace views of isovalue q for this CTA's block of a batch.
__device__ __forceinline__ FeIsoWs iso_ws(const FeWsAll& ws, int q) {
  FeIsoWs w = ws.iso[q];
  if (ws.stride) {
    const int64_t off = (int64_t)blockIdx.z * ws.stride;
    w.bits = shift_ptr(w.bits, off);
    w.sums = shift_ptr(w.sums, off);
    w.cnt = shift_ptr(w.cnt, off);
    w.wact = shift_ptr(w.wact, off);
    w.tot = shift_ptr(w.tot, off);
    w.rowoff = shift_ptr(w.rowoff, off);
    w.work = shift_ptr(w.work, off);
    w.ufirst = shift_ptr(w.ufirst, off);
    w.ucnt = shift_ptr(w.ucnt, off);
    w.wcnt = shift_ptr(w.wcnt, off);
    w.units = shift_ptr(w.units, off);
    w.flags = shift_ptr(w.flags, off);
    w.super = shift_ptr(w.super, off);
    w.agg = shift_ptr(w.agg, off);
    w.incl = shift_ptr(w.incl, off);
    w.info = shift_ptr(w.info, off);
  }
  return w;
}

// This CTA's block's mask, volume and geometry (the launch's own for one
// volume).
__device__ __forceinline__ const int32_t* block_mask(const FeWsAll& ws, const int32_t* mask) {
  return ws.vols ? (ws.masks ? ws.masks[blockIdx.z] : nullptr) : mask;
}
__device__ __forceinline__ const float* block_vol(const FeWsAll& ws, const float* v) {
  return ws.vols ? ws.vols[blockIdx.z] : v;
}
__device__ __forceinline__ const float* block_geom(const FeWsAll& ws, const float* g) {
  return ws.geoms ? ws.geoms + 6 * (int64_t)blockIdx.z : g;
}

// Bits of four node rows around one word: a = (j,k), b = (j+1,k),
// c = (j,k+1), d = (j+1,k+1), each with the next word's bit 0 available
// through the *n values.
struct Quad {
  uint32_t a, b, c, d, an, bn, cn, dn;
};

// Lanes sl of one S-lane row segment hold words w = w0 + sl.  Fills the next
// word of each row from the neighbouring lane, or loads it at the segment end.
__device__ __forceinline__ void load_quad(Quad& q, const uint32_t* __restrict__ bits,
                                          const FeDims& d, int S, int64_t rowbit, int w,
                                          int sl, bool valid, bool hasY, bool hasZ) {
  const int64_t L = d.L;
  const int64_t plane = d.L * d.M;
  const bool hasC = hasY && hasZ;
  q.a = valid ? row_word(bits, rowbit, w, L) : 0u;
  q.b = hasY ? row_word(bits, rowbit + L, w, L) : 0u;
  q.c = hasZ ? row_word(bits, rowbit + plane, w, L) : 0u;
  q.d = hasC ? row_word(bits, rowbit + plane + L, w, L) : 0u;
  q.an = __shfl_down_sync(0xffffffffu, q.a, 1, S);
  q.bn = __shfl_down_sync(0xffffffffu, q.b, 1, S);
  q.cn = __shfl_down_sync(0xffffffffu, q.c, 1, S);
  q.dn = __shfl_down_sync(0xffffffffu, q.d, 1, S);
  if (sl == S - 1) {
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
// K2: per-row counts (K2a), then a single-pass scan of them (K2b)
// ------------------------------------------------------------------------

// Triangles of the (up to 32) cells of one word, bit-parallel.  For every
// case of the marching-cubes table, triangles = V - 2F - 4*belt + 4*full,
// where V counts corners above the isovalue, F the faces with all four
// corners above, belt is 1 when exactly two antipodal corners are below, and
// full is 1 when all eight are above.  (It is #cut edges - 2 * #components
// of the above corners, with the cube graph's two kinds of non-face cycles
// corrected; checked against all 256 table entries.)  Corner words:
// 0 a, 1 a1, 2 b1, 3 b, 4 c, 5 c1, 6 d1, 7 d; xm selects the valid cells.
__device__ __forceinline__ unsigned tri_count_word(uint32_t a, uint32_t a1, uint32_t b,
                                                   uint32_t b1, uint32_t c, uint32_t c1,
                                                   uint32_t d, uint32_t d1, uint32_t xm) {
  const unsigned V = __popc(a & xm) + __popc(a1 & xm) + __popc(b & xm) + __popc(b1 & xm) +
                     __popc(c & xm) + __popc(c1 & xm) + __popc(d & xm) + __popc(d1 & xm);
  const uint32_t ab = a & b, a1b1 = a1 & b1, cd = c & d, c1d1 = c1 & d1;
  const uint32_t f0 = ab & a1b1;        // corners 0 1 2 3
  const uint32_t f1 = cd & c1d1;        // 4 5 6 7
  const uint32_t f2 = a & a1 & c & c1;  // 0 1 5 4
  const uint32_t f3 = b & b1 & d & d1;  // 3 2 6 7
  const uint32_t f4 = ab & cd;          // 0 3 7 4
  const uint32_t f5 = a1b1 & c1d1;      // 1 2 6 5
  const unsigned F = __popc(f0 & xm) + __popc(f1 & xm) + __popc(f2 & xm) + __popc(f3 & xm) +
                     __popc(f4 & xm) + __popc(f5 & xm);
  const uint32_t full = f0 & f1 & xm;
  const uint32_t belt = (~a & ~d1 & a1 & b1 & b & c & c1 & d) |   // 0 and 6 below
                        (~a1 & ~d & a & b1 & b & c & c1 & d1) |   // 1 and 7
                        (~b1 & ~c & a & a1 & b & c1 & d1 & d) |   // 2 and 4
                        (~b & ~c1 & a & a1 & b1 & c & d1 & d);    // 3 and 5
  return V - 2 * F - 4 * __popc(belt & xm) + 4 * __popc(full);
}

// K2a: per-row counts {X, Y, Z, T} of one tile of TR rows -> cnt[R][4],
// and per-row word-activity masks -> wact[R][AW].  Tiles are independent.
//
// The tile's bit rows [R0, R0+TR] and their next-plane neighbours
// [R0+M, R0+M+TR] are each one contiguous run of the flat bitmask; both are
// copied to shared memory with 16-byte cp.async (all copies in flight at
// once).  A row is then handled by an S-lane segment, one word per lane
// (S = 32 for rows of >= 1024 nodes, fewer for short rows, which then share
// a warp).  Warps whose rows have no side change anywhere skip the word
// arithmetic entirely; the surface is sparse, so most rows do.

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Copy bitmask words [first, first + words) into s with 16-byte cp.async
// copies from the 16-byte boundary at or below `first`; returns the index in
// s of word `first`.  The bitmask has >= 8 zero padding words, so the
// rounded-up tail stays inside the allocation.
__device__ __forceinline__ int stage_run(uint32_t* s, const uint32_t* bits, int64_t first,
                                         int64_t words) {
  const int64_t g0 = first & ~(int64_t)3;
  const int shift = (int)(first - g0);
  const int64_t nvec = (shift + words + 3) >> 2;
  for (int64_t i = threadIdx.x; i < nvec; i += kThreads) cp_async16(s + 4 * i, bits + g0 + 4 * i);
  return shift;
}

// Word w of the row whose first node is bit b of the staged run s (zero
// beyond the row's length L), and bit 0 of word w + 1 in *next0.
__device__ __forceinline__ uint32_t staged_word(const uint32_t* s, int b, int w, int L,
                                                uint32_t* next0) {
  const int rem = L - 32 * w;
  if (rem <= 0) {
    *next0 = 0u;
    return 0u;
  }
  const int pos = b + 32 * w;
  const int q = pos >> 5, sh = pos & 31;
  const uint32_t lo = s[q], hi = s[q + 1];
  uint32_t x = sh ? __funnelshift_r(lo, hi, sh) : lo;
  *next0 = rem > 32 ? (hi >> sh) & 1u : 0u;
  if (rem < 32) x &= (1u << rem) - 1u;
  return x;
}

// Words per staged run: the run, the 16-byte alignment shift in front of it
// and the rounding of the last 16-byte copy.
__host__ __device__ __forceinline__ int64_t k2_stage_words(int TR, int W) {
  return (((int64_t)(TR + 1) * W + 3 + 8) + 3) & ~(int64_t)3;
}

// Rows of one K2a tile, ALIGNED = every row starts on a word (L % 32 == 0).
template <bool ALIGNED>
__device__ __forceinline__ void count_rows(const FeDims& d, const FeIsoWs& Wk,
                                           const int32_t* __restrict__ mask, const int* s_ntri,
                                           const uint32_t* sAr, const uint32_t* sCr,
                                           int64_t R0, int64_t a_first, int64_t c_first) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int S = d.S, logS = d.logS, G = 32 >> logS;
  const int seg = lane >> logS, sl = lane & (S - 1);
  const int W = d.W, TR = d.TR;
  const int64_t L = d.L;
  const int Li = (int)L;
  const uint32_t M32 = (uint32_t)d.M;
  const int passes = (TR + 8 * G - 1) / (8 * G);
  // Row of pass 0, then advance by 8G rows per pass without dividing.
  const int local0 = warp * G + seg;
  uint32_t j = (uint32_t)(R0 + local0) % M32, k = (uint32_t)(R0 + local0) / M32;
  const uint32_t step = 8u * (uint32_t)G, dj = step % M32, dk = step / M32;
  for (int p = 0; p < passes; ++p) {
    const int local = local0 + p * (int)step;
    if (p > 0) {
      j += dj;
      k += dk;
      if (j >= M32) { j -= M32; ++k; }
    }
    const int64_t r = R0 + local;
    const bool valid = local < TR && r < d.R;
    const bool hasY = valid && (j + 1 < M32);
    const bool hasZ = valid && ((int64_t)k + 1 < d.N);
    const bool hasC = hasY && hasZ;
    const int ba = (int)(r * L - a_first * 32), bb = ba + Li;
    const int bc = (int)((r + d.M) * L - c_first * 32), bd = bc + Li;
    unsigned cX = 0, cY = 0, cZ = 0, cT = 0;
    bool any = false;
    for (int w0 = 0; w0 < W; w0 += S) {
      const int w = w0 + sl;
      uint32_t a = 0, an = 0, b, bn, c, cn, dd, dn;
      if (ALIGNED) {
        const bool in = w < W, more = w + 1 < W;
        if (valid && in) { a = sAr[(ba >> 5) + w]; an = more ? (sAr[(ba >> 5) + w + 1] & 1u) : 0u; }
        if (hasY && in) { b = sAr[(bb >> 5) + w]; bn = more ? (sAr[(bb >> 5) + w + 1] & 1u) : 0u; }
        else { b = a; bn = an; }
        if (hasZ && in) { c = sCr[(bc >> 5) + w]; cn = more ? (sCr[(bc >> 5) + w + 1] & 1u) : 0u; }
        else { c = a; cn = an; }
        if (hasC && in) { dd = sCr[(bd >> 5) + w]; dn = more ? (sCr[(bd >> 5) + w + 1] & 1u) : 0u; }
        else { dd = b; dn = bn; }
      } else {
        if (valid) a = staged_word(sAr, ba, w, Li, &an);
        // A missing neighbour row reads as a copy of row a (no crossings).
        if (hasY) b = staged_word(sAr, bb, w, Li, &bn); else { b = a; bn = an; }
        if (hasZ) c = staged_word(sCr, bc, w, Li, &cn); else { c = a; cn = an; }
        if (hasC) dd = staged_word(sCr, bd, w, Li, &dn); else { dd = b; dn = bn; }
      }
      const uint32_t a1 = (a >> 1) | (an << 31);
      const uint32_t u = (a ^ b) | (a ^ c) | (a ^ dd);
      const uint32_t un = (an ^ bn) | (an ^ cn) | (an ^ dn);
      const bool busy = ((u | (a ^ a1) | (un << 31)) & low_mask(Li - 32 * w)) != 0u;
      // Warps with no side change in any of their rows skip the arithmetic.
      const uint32_t bal = __ballot_sync(0xffffffffu, busy);
      uint32_t amask = 0;
      if (bal != 0u) {
        any = true;
        unsigned x0 = 0, y0 = 0, z0 = 0, t0 = 0;
        if (busy) {
          const uint32_t xm = low_mask(Li - 1 - 32 * w);
          x0 = __popc((a ^ a1) & xm);
          y0 = __popc(a ^ b);
          z0 = __popc(a ^ c);
          if (hasC) {
            const uint32_t b1 = (b >> 1) | (bn << 31), c1 = (c >> 1) | (cn << 31);
            const uint32_t d1 = (dd >> 1) | (dn << 31);
            t0 = tri_count_word(a, a1, b, b1, c, c1, dd, d1, xm);
            if (mask) {  // masked cells emit nothing: take their triangles back out
              const int64_t cell_row0 = ((int64_t)k * d.ny + j) * d.nx;
              uint32_t act = (u | (u >> 1) | (un << 31) | (a ^ a1)) & xm;
              while (act) {
                const int bit = __ffs(act) - 1;
                act &= act - 1;
                if (__ldg(mask + cell_row0 + 32 * w + bit) != 0)
                  t0 -= s_ntri[cell_case(bit, a, a1, b, b1, c, c1, dd, d1)];
              }
            }
          }
          cX += x0;
          cY += y0;
          cZ += z0;
          cT += t0;
        }
        // Activity bits of words [w0, w0 + S) of this segment's row.  Either
        // the row fits one segment (w0 == 0) or S == 32, so each chunk owns
        // exactly one mask word.
        amask = (__ballot_sync(0xffffffffu, (x0 | y0 | z0 | t0) != 0u) >> (seg << logS)) &
                low_mask(S);
      }
      if (sl == 0 && valid) Wk.wact[r * d.AW + (w0 >> 5)] = amask;
    }
    if (any) {  // row totals over the segment (all zero otherwise)
      for (int o = S >> 1; o > 0; o >>= 1) {
        cX += __shfl_xor_sync(0xffffffffu, cX, o);
        cY += __shfl_xor_sync(0xffffffffu, cY, o);
        cZ += __shfl_xor_sync(0xffffffffu, cZ, o);
        cT += __shfl_xor_sync(0xffffffffu, cT, o);
      }
    }
    if (sl == 0 && valid)
      reinterpret_cast<int4*>(Wk.cnt)[r] = make_int4((int)cX, (int)cY, (int)cZ, (int)cT);
  }
}

__global__ void __launch_bounds__(kThreads, 3)
k_fe_count(FeDims d, FeWsAll ws, const int32_t* __restrict__ mask, int64_t nwords) {
  extern __shared__ uint32_t k2_smem[];
  __shared__ int s_ntri[256];
  const FeIsoWs Wk = iso_ws(ws, blockIdx.y);
  const int32_t* __restrict__ mask_b = block_mask(ws, mask);
  const int tid = threadIdx.x;
  const int TR = d.TR, W = d.W;
  const int64_t stage = k2_stage_words(TR, W);
  uint32_t* sA = k2_smem;
  uint32_t* sC = k2_smem + stage;
  s_ntri[tid] = (int)(c_case_tris[tid] >> 60);
  const int64_t R0 = (int64_t)blockIdx.x * TR;
  const int64_t L = d.L;

  const int64_t a_first = (R0 * L) >> 5;
  const int64_t a_last_row = min(R0 + TR + 1, d.R);
  const int64_t a_words = min(((a_last_row * L + 31) >> 5) + 1, nwords + 1) - a_first;
  const uint32_t* sAr = sA + stage_run(sA, Wk.bits, a_first, a_words);
  const int64_t c_row0 = R0 + d.M;
  int64_t c_first = 0;
  const uint32_t* sCr = sC;
  if (c_row0 < d.R) {
    c_first = (c_row0 * L) >> 5;
    const int64_t c_last_row = min(c_row0 + TR + 1, d.R);
    const int64_t c_words = min(((c_last_row * L + 31) >> 5) + 1, nwords + 1) - c_first;
    sCr = sC + stage_run(sC, Wk.bits, c_first, c_words);
  }
  cp_async_wait_all();
  __syncthreads();
  if ((L & 31) == 0)
    count_rows<true>(d, Wk, mask_b, s_ntri, sAr, sCr, R0, a_first, c_first);
  else
    count_rows<false>(d, Wk, mask_b, s_ntri, sAr, sCr, R0, a_first, c_first);
}

// Position of the k-th (0-based) set bit of m; k < popc(m).
__device__ __forceinline__ int nth_set_bit(uint32_t m, int k) {
  int pos = 0;
#pragma unroll
  for (int sft = 16; sft >= 1; sft >>= 1) {
    const int low = __popc(m & ((1u << sft) - 1u));
    if (k >= low) {
      k -= low;
      m >>= sft;
      pos += sft;
    }
  }
  return pos;
}

// Exclusive prefix of `x` over the lanes of the caller's run, where runs are
// maximal sequences of lanes with equal `key` (keys of a run are contiguous).
// *run_total receives the run's total in the run's last lane.
__device__ __forceinline__ unsigned seg_excl(unsigned x, int key, unsigned* run_total,
                                             bool* is_last) {
  const int lane = threadIdx.x & 31;
  unsigned incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const int prev = __shfl_up_sync(0xffffffffu, key, 1);
  const bool head = lane == 0 || prev != key;
  const uint32_t hm = __ballot_sync(0xffffffffu, head);
  const int first = 31 - __clz(hm & (lane == 31 ? 0xffffffffu : ((2u << lane) - 1u)));
  const unsigned before = __shfl_sync(0xffffffffu, incl, first > 0 ? first - 1 : 0);
  const unsigned base = first > 0 ? before : 0u;
  *is_last = lane == 31 || ((hm >> (lane + 1)) & 1u);
  *run_total = incl - base;
  return incl - x - base;
}

// Word-aligned rows (L % 32 == 0): counts, offsets and the unit list.
//
// One thread per node row.  For each group of 32 words of its row the
// thread reads K1's {mixed, ones} summaries of the four rows around its
// cells (8 bytes each) and forms the candidate words: a word can hold a
// crossing or a cut cell only if one of the four rows is mixed there or at
// the next word, or the rows' uniform values differ there or at the next
// word, or row a's uniform value changes at the next word.  Only candidates
// are loaded from the bitmask and counted exactly as the reference counts
// them; on a smooth surface they are a few percent of all words.
//
// A word with any output (own x/y/z crossings or triangles) is a "unit".
// Three launches with no waiting between blocks: K2a counts (rows, words,
// units) and leaves per-tile totals, K2b scans the tiles' totals, K2c writes
// each row's offsets, the index of its first unit, and one FeUnit per unit
// holding the section-relative offsets of the word's first x, y, z point and
// first triangle.  Units are in (row, word) order, so the first unit at or
// after any (row, word) position carries the offsets a crossing there would
// have; the emit kernel finds neighbour rows' offsets that way.

// Summary bits of flat words [f, f + 33) (the 33rd is word f + 32).
__device__ __forceinline__ void sum_window(const uint2* __restrict__ s, int64_t f,
                                           uint64_t* mixed, uint64_t* ones) {
  const int64_t c = f >> 5;
  const int o = (int)(f & 31);
  const uint2 lo = __ldg(s + c), hi = __ldg(s + c + 1);
  *mixed = (((((uint64_t)hi.x) << 32) | lo.x) >> o) & 0x1ffffffffull;
  *ones = (((((uint64_t)hi.y) << 32) | lo.y) >> o) & 0x1ffffffffull;
}

// First flat words of the four rows around node row r (aligned rows).  A
// missing neighbour row reads as a copy of row a (b, c) or of row b (d), so
// it adds no crossings.
struct RowQuad {
  int64_t fa, fb, fc, fd;
  uint32_t j, k;
  bool hasY, hasZ, hasC;
};

__device__ __forceinline__ RowQuad row_quad(const FeDims& d, int64_t r) {
  RowQuad q;
  const uint32_t M32 = (uint32_t)d.M;
  q.j = (uint32_t)r % M32;
  q.k = (uint32_t)r / M32;
  q.hasY = q.j + 1 < M32;
  q.hasZ = (int64_t)q.k + 1 < d.N;
  q.hasC = q.hasY && q.hasZ;
  q.fa = r * d.W;
  q.fb = q.hasY ? q.fa + d.W : q.fa;
  q.fc = q.hasZ ? q.fa + d.M * d.W : q.fa;
  q.fd = q.hasC ? q.fc + d.W : q.fb;
  return q;
}

// Candidate words of group g (words 32g .. 32g+31) of the row.
__device__ __forceinline__ uint32_t candidates(const uint2* __restrict__ sums, const RowQuad& q,
                                               int W, int g) {
  const int w0 = 32 * g;
  const int nvalid = W - w0;  // words of the row in this group (>= 1)
  const uint64_t vm = nvalid >= 32 ? 0xffffffffull : ((1ull << nvalid) - 1ull);
  const uint64_t nm = nvalid - 1 >= 32 ? 0xffffffffull : ((1ull << (nvalid - 1)) - 1ull);
  uint64_t ma, oa, mb, ob, mc, oc, md, od;
  sum_window(sums, q.fa + w0, &ma, &oa);
  sum_window(sums, q.fb + w0, &mb, &ob);
  sum_window(sums, q.fc + w0, &mc, &oc);
  sum_window(sums, q.fd + w0, &md, &od);
  const uint64_t x = ma | mb | mc | md | (oa ^ ob) | (oa ^ oc) | (oa ^ od);
  return (uint32_t)((x | (((x >> 1) | (oa ^ (oa >> 1))) & nm)) & vm);
}

// The bit words of the four rows at word w, and bit 0 of word w + 1 (zero
// past the row's end).
struct WordQuad {
  uint32_t a, b, c, d, an, bn, cn, dn;
};

__device__ __forceinline__ WordQuad load_word_quad(const uint32_t* __restrict__ bits,
                                                   const RowQuad& q, int w, int W) {
  WordQuad x;
  x.a = __ldg(bits + q.fa + w);
  x.b = __ldg(bits + q.fb + w);
  x.c = __ldg(bits + q.fc + w);
  x.d = __ldg(bits + q.fd + w);
  x.an = x.bn = x.cn = x.dn = 0u;
  if (w + 1 < W) {
    x.an = __ldg(bits + q.fa + w + 1) & 1u;
    x.bn = __ldg(bits + q.fb + w + 1) & 1u;
    x.cn = __ldg(bits + q.fc + w + 1) & 1u;
    x.dn = __ldg(bits + q.fd + w + 1) & 1u;
  }
  return x;
}

// Exact counts of word w: own x, y, z crossings and triangles of its cells
// (masked cells emit none), packed as x | y << 6 | z << 12 | t << 18.
__device__ __forceinline__ uint32_t count_word(const WordQuad& x, const RowQuad& q, int w, int Li,
                                               const FeDims& d, const int32_t* __restrict__ mask,
                                               const int* s_ntri) {
  const uint32_t a1 = (x.a >> 1) | (x.an << 31);
  const uint32_t xm = low_mask(Li - 1 - 32 * w);
  const unsigned x0 = __popc((x.a ^ a1) & xm);
  const unsigned y0 = __popc(x.a ^ x.b);
  const unsigned z0 = __popc(x.a ^ x.c);
  unsigned t0 = 0;
  if (q.hasC) {
    const uint32_t b1 = (x.b >> 1) | (x.bn << 31), c1 = (x.c >> 1) | (x.cn << 31);
    const uint32_t d1 = (x.d >> 1) | (x.dn << 31);
    t0 = tri_count_word(x.a, a1, x.b, b1, x.c, c1, x.d, d1, xm);
    if (mask && t0) {  // masked cells emit nothing: take their triangles back out
      const int64_t cell_row0 = ((int64_t)q.k * d.ny + q.j) * d.nx;
      const uint32_t uu = (x.a ^ x.b) | (x.a ^ x.c) | (x.a ^ x.d);
      const uint32_t un = (x.an ^ x.bn) | (x.an ^ x.cn) | (x.an ^ x.dn);
      uint32_t act = (uu | (uu >> 1) | (un << 31) | (x.a ^ a1)) & xm;
      while (act) {
        const int bit = __ffs(act) - 1;
        act &= act - 1;
        if (__ldg(mask + cell_row0 + 32 * w + bit) != 0)
          t0 -= (unsigned)s_ntri[cell_case(bit, x.a, a1, x.b, b1, x.c, c1, x.d, d1)];
      }
    }
  }
  return x0 | (y0 << 6) | (z0 << 12) | (t0 << 18);
}

constexpr int kSuperTiles = 64;  // count tiles per super-tile total

__device__ __forceinline__ void put_unit(FeUnit* units, int64_t cap, int64_t ui, uint32_t r,
                                         uint32_t w, const long long (&o)[4]) {
  if (ui >= cap) return;  // cannot happen: the list holds every word and the sentinel
  uint4* p = reinterpret_cast<uint4*>(units + ui);
  p[0] = make_uint4(r, w, (uint32_t)o[0], (uint32_t)o[1]);
  p[1] = make_uint4((uint32_t)o[2], 0u, (uint32_t)(unsigned long long)o[3],
                    (uint32_t)((unsigned long long)o[3] >> 32));
}

// Largest lane l whose (non-decreasing across lanes) value v_l is <= e.
__device__ __forceinline__ int owner_lane(unsigned v, unsigned e) {
  int lo = 0;
#pragma unroll
  for (int step = 16; step >= 1; step >>= 1) {
    const unsigned vm = __shfl_sync(0xffffffffu, v, lo + step < 32 ? lo + step : 31);
    if (lo + step < 32 && vm <= e) lo += step;
  }
  return lo;
}

// K2a (word-aligned rows): per-row counts, activity masks and per-word
// counts.  A warp owns 32 consecutive node rows.  Lane = row finds the row's
// candidate words; the warp then lists all candidates of its rows and counts
// them 32 at a time, lane = candidate, so that the bit loads of 32 words are
// in flight together.  Per-row sums go through shared-memory atomics; each
// active word's packed counts are kept (wcnt) for the offsets pass.  Each
// block also leaves its tile's totals {X, Y, Z, T, units} and adds them to
// its super-tile's.
__global__ void __launch_bounds__(kThreads)
k_fe_count_words(FeDims d, FeWsAll ws, const int32_t* __restrict__ mask) {
  __shared__ int s_ntri[256];
  __shared__ unsigned s_cnt[4][kThreads];
  __shared__ unsigned s_nu[kThreads];
  __shared__ uint32_t s_act[kThreads];
  const FeIsoWs Wk = iso_ws(ws, blockIdx.y);
  const int32_t* __restrict__ mask_b = block_mask(ws, mask);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  griddep_launch();
  s_ntri[tid] = (int)(c_case_tris[tid] >> 60);  // kThreads == 256
#pragma unroll
  for (int t = 0; t < 4; ++t) s_cnt[t][tid] = 0;
  s_nu[tid] = 0;
  griddep_wait();  // the bitmask and summaries of the threshold pass
  __syncthreads();
  const int64_t rbase = (int64_t)blockIdx.x * kThreads + warp * 32;  // the warp's first row
  const int64_t r = rbase + lane;
  const bool valid = r < d.R;
  const int W = d.W, Li = (int)d.L;
  RowQuad q{};
  if (valid) q = row_quad(d, r);
  for (int g = 0; g < d.AW; ++g) {
    const uint32_t cand = valid ? candidates(Wk.sums, q, W, g) : 0u;
    s_act[tid] = 0u;
    const unsigned nc = __popc(cand);
    unsigned pre = nc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, pre, o);
      if (lane >= o) pre += y;
    }
    const unsigned NC = __shfl_sync(0xffffffffu, pre, 31);
    pre -= nc;
    __syncwarp();
    for (unsigned b0 = 0; b0 < NC; b0 += 32) {
      const unsigned e = b0 + lane;
      const bool ve = e < NC;
      const int own = owner_lane(pre, ve ? e : NC - 1);
      const uint32_t ocand = __shfl_sync(0xffffffffu, cand, own);
      const unsigned opre = __shfl_sync(0xffffffffu, pre, own);
      // The owner row's geometry from the owner lane (no division here).
      RowQuad oq;
      oq.fa = __shfl_sync(0xffffffffu, q.fa, own);
      oq.j = __shfl_sync(0xffffffffu, q.j, own);
      oq.k = __shfl_sync(0xffffffffu, q.k, own);
      const unsigned oflags = __shfl_sync(0xffffffffu, (q.hasY ? 1u : 0u) | (q.hasZ ? 2u : 0u), own);
      uint32_t c = 0u;
      int w = 0;
      if (ve) {
        const int wb = nth_set_bit(ocand, (int)(e - opre));
        w = 32 * g + wb;
        oq.hasY = (oflags & 1u) != 0;
        oq.hasZ = (oflags & 2u) != 0;
        oq.hasC = oflags == 3u;
        oq.fb = oq.hasY ? oq.fa + W : oq.fa;
        oq.fc = oq.hasZ ? oq.fa + d.M * W : oq.fa;
        oq.fd = oq.hasC ? oq.fc + W : oq.fb;
        c = count_word(load_word_quad(Wk.bits, oq, w, W), oq, w, Li, d, mask_b, s_ntri);
      }
      if (c != 0u) {
        const int rl = warp * 32 + own;
        atomicAdd(&s_cnt[0][rl], c & 63u);
        atomicAdd(&s_cnt[1][rl], (c >> 6) & 63u);
        atomicAdd(&s_cnt[2][rl], (c >> 12) & 63u);
        atomicAdd(&s_cnt[3][rl], c >> 18);
        atomicOr(&s_act[rl], 1u << (w & 31));
        Wk.wcnt[(rbase + own) * W + w] = c;
      }
    }
    __syncwarp();
    if (valid) {
      Wk.wact[r * d.AW + g] = s_act[tid];
      s_nu[tid] += __popc(s_act[tid]);
    }
    __syncwarp();
  }
  long long own5[5] = {0, 0, 0, 0, 0};
  if (valid) {
    reinterpret_cast<int4*>(Wk.cnt)[r] =
        make_int4((int)s_cnt[0][tid], (int)s_cnt[1][tid], (int)s_cnt[2][tid], (int)s_cnt[3][tid]);
    Wk.ucnt[r] = s_nu[tid];
#pragma unroll
    for (int t = 0; t < 4; ++t) own5[t] = s_cnt[t][tid];
    own5[4] = s_nu[tid];
  }
  // Each warp adds its rows' totals to the tile's and the super-tile's (both
  // zeroed before the pass): no block barrier, warps leave as they finish.
#pragma unroll
  for (int t = 0; t < 5; ++t) {
    long long x = own5[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == t && x != 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(Wk.agg + blockIdx.x * 5 + t),
                (unsigned long long)x);
      atomicAdd(reinterpret_cast<unsigned long long*>(Wk.super + (blockIdx.x / kSuperTiles) * 5 + t),
                (unsigned long long)x);
    }
  }
}

// K2a with the candidate words of the whole block shared by its 256 threads
// (word-aligned rows, grids of few blocks: the small slabs of several GPUs).
// The rows' candidates are listed block-wide (a block prefix of the per-row
// counts in shared memory, with each row's geometry), then thread = candidate
// over the whole list, so the block takes as long as its average warp rather
// than its busiest one: one warp's 32 rows can hold most of the block's
// surface.  Same outputs as k_fe_count_words.
__global__ void __launch_bounds__(kThreads)
k_fe_count_words_bal(FeDims d, FeWsAll ws, const int32_t* __restrict__ mask) {
  __shared__ int s_ntri[256];
  __shared__ unsigned s_cnt[4][kThreads];
  __shared__ unsigned s_nu[kThreads];
  __shared__ uint32_t s_act[kThreads];
  __shared__ uint32_t s_cand[kThreads];
  __shared__ unsigned s_pre[kThreads];
  __shared__ unsigned s_wsum[kThreads / 32];
  __shared__ long long s_fa[kThreads];
  __shared__ uint32_t s_j[kThreads], s_k[kThreads], s_fl[kThreads];
  const FeIsoWs Wk = iso_ws(ws, blockIdx.y);
  const int32_t* __restrict__ mask_b = block_mask(ws, mask);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  griddep_launch();
  s_ntri[tid] = (int)(c_case_tris[tid] >> 60);  // kThreads == 256
#pragma unroll
  for (int t = 0; t < 4; ++t) s_cnt[t][tid] = 0;
  s_nu[tid] = 0;
  griddep_wait();  // the bitmask and summaries of the threshold pass
  const int64_t rbase = (int64_t)blockIdx.x * kThreads;  // the block's first row
  const int64_t r = rbase + tid;
  const bool valid = r < d.R;
  const int W = d.W, Li = (int)d.L;
  RowQuad q{};
  if (valid) q = row_quad(d, r);
  s_fa[tid] = q.fa;
  s_j[tid] = q.j;
  s_k[tid] = q.k;
  s_fl[tid] = (q.hasY ? 1u : 0u) | (q.hasZ ? 2u : 0u);
  for (int g = 0; g < d.AW; ++g) {
    const uint32_t cand = valid ? candidates(Wk.sums, q, W, g) : 0u;
    const unsigned nc = __popc(cand);
    unsigned pre = nc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, pre, o);
      if (lane >= o) pre += y;
    }
    if (lane == 31) s_wsum[warp] = pre;
    s_cand[tid] = cand;
    s_act[tid] = 0u;
    __syncthreads();
    unsigned before = 0, NC = 0;
#pragma unroll
    for (int w2 = 0; w2 < kThreads / 32; ++w2) {
      const unsigned x = s_wsum[w2];
      before += w2 < warp ? x : 0u;
      NC += x;
    }
    s_pre[tid] = before + pre - nc;  // block-exclusive prefix of the row's candidates
    __syncthreads();
    for (unsigned e = tid; e < NC; e += kThreads) {
      // The row holding candidate e: the last row whose prefix is <= e (rows
      // without candidates share the prefix of the next row that has some).
      int own = 0;
#pragma unroll
      for (int step = kThreads / 2; step >= 1; step >>= 1)
        if (s_pre[own + step] <= e) own += step;
      const int wb = nth_set_bit(s_cand[own], (int)(e - s_pre[own]));
      const int w = 32 * g + wb;
      RowQuad oq;
      oq.fa = s_fa[own];
      oq.j = s_j[own];
      oq.k = s_k[own];
      const uint32_t fl = s_fl[own];
      oq.hasY = (fl & 1u) != 0;
      oq.hasZ = (fl & 2u) != 0;
      oq.hasC = fl == 3u;
      oq.fb = oq.hasY ? oq.fa + W : oq.fa;
      oq.fc = oq.hasZ ? oq.fa + d.M * W : oq.fa;
      oq.fd = oq.hasC ? oq.fc + W : oq.fb;
      const uint32_t c = count_word(load_word_quad(Wk.bits, oq, w, W), oq, w, Li, d, mask_b, s_ntri);
      if (c != 0u) {
        atomicAdd(&s_cnt[0][own], c & 63u);
        atomicAdd(&s_cnt[1][own], (c >> 6) & 63u);
        atomicAdd(&s_cnt[2][own], (c >> 12) & 63u);
        atomicAdd(&s_cnt[3][own], c >> 18);
        atomicOr(&s_act[own], 1u << (w & 31));
        Wk.wcnt[(rbase + own) * W + w] = c;
      }
    }
    __syncthreads();
    if (valid) {
      Wk.wact[r * d.AW + g] = s_act[tid];
      s_nu[tid] += __popc(s_act[tid]);
    }
    __syncthreads();
  }
  long long own5[5] = {0, 0, 0, 0, 0};
  if (valid) {
    reinterpret_cast<int4*>(Wk.cnt)[r] =
        make_int4((int)s_cnt[0][tid], (int)s_cnt[1][tid], (int)s_cnt[2][tid], (int)s_cnt[3][tid]);
    Wk.ucnt[r] = s_nu[tid];
#pragma unroll
    for (int t = 0; t < 4; ++t) own5[t] = s_cnt[t][tid];
    own5[4] = s_nu[tid];
  }
#pragma unroll
  for (int t = 0; t < 5; ++t) {
    long long x = own5[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == t && x != 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(Wk.agg + blockIdx.x * 5 + t),
                (unsigned long long)x);
      atomicAdd(reinterpret_cast<unsigned long long*>(Wk.super + (blockIdx.x / kSuperTiles) * 5 + t),
                (unsigned long long)x);
    }
  }
}

// K2b (word-aligned rows): the first unit of each row, the units and the
// totals (rows_only: the row offsets instead, for tkmc_fe_row_offsets).  The
// tile's prefix is the sum of the super-tile totals before its super-tile
// and of the tile totals before it within its super-tile; the grand totals
// are the sum of all super-tile totals; no block waits for another.  Lane =
// row for the offsets, then the warp writes its rows' units 32 at a time,
// lane = unit: the unit's word from the row's activity mask, its counts from
// wcnt, its offsets from the row's running offsets plus a segmented prefix
// over the batch.
__global__ void __launch_bounds__(kThreads)
k_fe_offsets_units(FeDims d, FeWsAll ws, int64_t unit_cap, int rows_only) {
  __shared__ long long s_w[5][kThreads / 32];
  __shared__ long long s_pre[5], s_all[5];
  __shared__ long long s_run[kThreads / 32][32][4];
  const FeIsoWs Wk = iso_ws(ws, blockIdx.y);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t tile = blockIdx.x;
  const int64_t rbase = tile * kThreads + warp * 32;  // the warp's first row
  const int64_t r = rbase + lane;
  const bool valid = r < d.R;
  griddep_launch();
  griddep_wait();  // the count pass's row counts and tile totals
  // The row's counts (and, for rows of one activity word, that word) are
  // loaded before the tile prefix, so both loads are in flight together.
  int4 c = make_int4(0, 0, 0, 0);
  unsigned nU = 0;
  uint32_t wa0 = 0;
  if (valid) {
    c = __ldcg(reinterpret_cast<const int4*>(Wk.cnt) + r);
    nU = __ldcg(Wk.ucnt + r);
    if (d.AW == 1 && !rows_only) wa0 = __ldcg(Wk.wact + r);
  }
  if (warp < 5) {  // warp k sums value k of the tile's prefix and of the grand total
    const int k = warp;
    const int64_t nsup = (d.ntiles + kSuperTiles - 1) / kSuperTiles, sup = tile / kSuperTiles;
    long long pre = 0, all = 0;
    for (int64_t i = lane; i < nsup; i += 32) {
      const long long x = (long long)__ldcg(Wk.super + i * 5 + k);
      all += x;
      if (i < sup) pre += x;
    }
    for (int64_t i = sup * kSuperTiles + lane; i < tile; i += 32) pre += __ldcg(Wk.agg + i * 5 + k);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      pre += __shfl_xor_sync(0xffffffffu, pre, o);
      all += __shfl_xor_sync(0xffffffffu, all, o);
    }
    if (lane == 0) {
      s_pre[k] = pre;
      s_all[k] = all;
    }
  }
  const long long own[5] = {c.x, c.y, c.z, c.w, nU};
  long long inc[5];
#pragma unroll
  for (int t = 0; t < 5; ++t) {
    long long x = own[t];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    inc[t] = x;
    if (lane == 31) s_w[t][warp] = x;
  }
  __syncthreads();
  long long ex[5];
#pragma unroll
  for (int t = 0; t < 5; ++t) {
    long long before = 0;
#pragma unroll
    for (int w2 = 0; w2 < kThreads / 32; ++w2)
      if (w2 < warp) before += s_w[t][w2];
    ex[t] = s_pre[t] + before + inc[t] - own[t];
  }
  if (rows_only) {
    if (valid) {
      longlong2* dst = reinterpret_cast<longlong2*>(Wk.rowoff + r * 4);
      dst[0] = make_longlong2(ex[0], ex[1]);
      dst[1] = make_longlong2(ex[2], ex[3]);
    }
    return;
  }
  if (valid) {
    Wk.ufirst[r] = (uint32_t)ex[4];
    // Own totals: the offsets of the first ghost row.
    if (r == d.n_own_rows) {
#pragma unroll
      for (int t = 0; t < 4; ++t) Wk.info[t] = Wk.tot[t] = ex[t];
      Wk.info[12] = ex[4];
    }
    if (r == 0) {
#pragma unroll
      for (int t = 0; t < 4; ++t) Wk.info[4 + t] = s_all[t];
      Wk.info[11] = s_all[4];
      if (d.n_own_rows == d.R) {
#pragma unroll
        for (int t = 0; t < 4; ++t) Wk.info[t] = Wk.tot[t] = s_all[t];
        Wk.info[12] = s_all[4];
      }
      // Sentinel after the last unit: the totals, for lookups past the end.
      const long long o[4] = {s_all[0], s_all[1], s_all[2], s_all[3]};
      put_unit(Wk.units, unit_cap, s_all[4], (uint32_t)d.R, 0u, o);
    }
  }
  // ---- the warp's units, lane = unit ----
#pragma unroll
  for (int t = 0; t < 4; ++t) s_run[warp][lane][t] = ex[t];
  unsigned pre = nU;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, pre, o);
    if (lane >= o) pre += y;
  }
  const unsigned NU = __shfl_sync(0xffffffffu, pre, 31);
  pre -= nU;
  const long long ufirst = ex[4];
  __syncwarp();
  for (unsigned b0 = 0; b0 < NU; b0 += 32) {
    const unsigned e = b0 + lane;
    const bool ve = e < NU;
    const int own_l = owner_lane(pre, ve ? e : NU - 1);
    const unsigned opre = __shfl_sync(0xffffffffu, pre, own_l);
    const long long ou = __shfl_sync(0xffffffffu, ufirst, own_l);
    const int64_t orow = rbase + own_l;
    int w = 0;
    uint32_t cw = 0;
    const uint32_t om = __shfl_sync(0xffffffffu, wa0, own_l);
    if (ve && d.AW == 1) {
      w = nth_set_bit(om, (int)(e - opre));
      cw = __ldcg(Wk.wcnt + orow * d.W + w);
    } else if (ve) {
      int k = (int)(e - opre);  // k-th active word of the row
      for (int i = 0; i < d.AW; ++i) {
        const uint32_t m = __ldcg(Wk.wact + orow * d.AW + i);
        const int n = __popc(m);
        if (k < n) {
          w = 32 * i + nth_set_bit(m, k);
          break;
        }
        k -= n;
      }
      cw = __ldcg(Wk.wcnt + orow * d.W + w);
    }
    const int key = ve ? own_l : -1;
    unsigned tA, tB;
    bool last;
    const unsigned xA = (cw & 63u) | (((cw >> 6) & 63u) << 11);
    const unsigned xB = ((cw >> 12) & 63u) | ((cw >> 18) << 11);
    const unsigned eA = seg_excl(xA, key, &tA, &last);
    const unsigned eB = seg_excl(xB, key, &tB, &last);
    if (ve) {
      const long long* rr = s_run[warp][own_l];
      const long long o[4] = {rr[0] + (eA & 2047u), rr[1] + (eA >> 11), rr[2] + (eB & 2047u),
                              rr[3] + (eB >> 11)};
      put_unit(Wk.units, unit_cap, ou + (long long)(e - opre), (uint32_t)orow, (uint32_t)w, o);
    }
    __syncwarp();
    if (ve && last) {
      long long* rr = s_run[warp][own_l];
      rr[0] += tA & 2047u;
      rr[1] += tA >> 11;
      rr[2] += tB & 2047u;
      rr[3] += tB >> 11;
    }
    __syncwarp();
  }
}

// K2b: single-pass (decoupled look-back) exclusive scan of the row counts
// into row offsets, totals and the worklist of active own rows.  A tile is
// kScanRows rows, 4 consecutive rows per thread.
constexpr int kScanRowsPerThread = 4;
constexpr int kScanRows = kThreads * kScanRowsPerThread;

__global__ void __launch_bounds__(kThreads)
k_fe_scan_rows(FeDims d, FeWsAll ws, int64_t wait_ns, int64_t skip_tile) {
  __shared__ long long s_wtot[4][kThreads / 32];
  __shared__ long long s_prefix[4];
  __shared__ int64_t s_tile;
  __shared__ unsigned s_wbase[kThreads / 32];
  const FeIsoWs W = iso_ws(ws, blockIdx.y);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_tile = (int64_t)atomicAdd((unsigned long long*)(W.info + 9), 1ull);
  __syncthreads();
  const int64_t tile = s_tile;
  const int64_t r0 = tile * kScanRows + (int64_t)tid * kScanRowsPerThread;

  int4 c[kScanRowsPerThread];
  long long own[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < kScanRowsPerThread; ++i) {
    c[i] = (r0 + i < d.R) ? __ldcg(reinterpret_cast<const int4*>(W.cnt) + r0 + i)
                          : make_int4(0, 0, 0, 0);
    own[0] += c[i].x; own[1] += c[i].y; own[2] += c[i].z; own[3] += c[i].w;
  }
  long long inc[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    long long x = own[q];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    inc[q] = x;
    if (lane == 31) s_wtot[q][warp] = x;
  }
  __syncthreads();
  long long tile_total[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    long long before = 0, all = 0;
#pragma unroll
    for (int w2 = 0; w2 < kThreads / 32; ++w2) {
      const long long t = s_wtot[q][w2];
      if (w2 < warp) before += t;
      all += t;
    }
    inc[q] += before;
    tile_total[q] = all;
  }
  if (warp == 0) {
    long long pre[4];
    lookback<4>(W.flags, W.agg, W.incl, tile, tile_total, pre, wait_ns, tile == skip_tile,
                W.info + 10);
    if (lane == 0)
#pragma unroll
      for (int q = 0; q < 4; ++q) s_prefix[q] = pre[q];
  }
  __syncthreads();

  long long ex[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) ex[q] = s_prefix[q] + inc[q] - own[q];
  unsigned act_bits = 0;
#pragma unroll
  for (int i = 0; i < kScanRowsPerThread; ++i) {
    const int64_t rr = r0 + i;
    if (rr < d.R) {
      longlong2* dst = reinterpret_cast<longlong2*>(W.rowoff + rr * 4);
      dst[0] = make_longlong2(ex[0], ex[1]);
      dst[1] = make_longlong2(ex[2], ex[3]);
      // Own totals: the offset of the first ghost row, or the grand total.
      if (rr == d.n_own_rows)
#pragma unroll
        for (int q = 0; q < 4; ++q) W.info[q] = W.tot[q] = ex[q];
      if (rr < d.n_own_rows && (c[i].x | c[i].y | c[i].z | c[i].w) != 0) act_bits |= 1u << i;
    }
    ex[0] += c[i].x; ex[1] += c[i].y; ex[2] += c[i].z; ex[3] += c[i].w;
    if (rr == d.R - 1) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        W.info[4 + q] = ex[q];
        if (d.n_own_rows == d.R) W.info[q] = W.tot[q] = ex[q];
      }
    }
  }
  // Worklist of own rows with any output (order is irrelevant: every row
  // writes at its own offsets).
  const unsigned nact = __popc(act_bits);
  unsigned incl_n = nact;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, incl_n, o);
    if (lane >= o) incl_n += y;
  }
  const unsigned wtotal = __shfl_sync(0xffffffffu, incl_n, 31);
  if (lane == 31 && wtotal)
    s_wbase[warp] = (unsigned)atomicAdd((unsigned long long*)(W.info + 8),
                                        (unsigned long long)wtotal);
  __syncwarp();
  if (nact) {
    unsigned pos = s_wbase[warp] + incl_n - nact;
    for (int i = 0; i < kScanRowsPerThread; ++i)
      if (act_bits & (1u << i)) W.work[pos++] = (uint32_t)(r0 + i);
  }
}

// ------------------------------------------------------------------------
// K3: emit points and triangles of the active rows
// ------------------------------------------------------------------------
//
// Phase 1 (lane = one 32-node word of a row, S lanes per row): load the four
// bit rows around the word, form the crossing masks and the active-cell mask,
// and scan the per-word crossing counts across the row.  Each word's masks,
// bits and absolute offsets go to a shared-memory record.
// Phase 2 (lane = one node/cell of a word): loop over the words with output;
// all 32 lanes emit that word together -- one coalesced 128-byte read of the
// row's values, contiguous point stores, and one triangle scan per word.

struct FeEmitArgs {
  const float* v;
  const int32_t* mask;
  float* points;
  int32_t* conn;
  long long points_cap, conn_cap;  // rows of 3
  float geom[6];
  int64_t k_offset;
  IsoParams iso;
  long long pt_id_base[TKMC_MAX_ISO][3];
  long long pt_out_base[TKMC_MAX_ISO][3];
  long long tri_out_base[TKMC_MAX_ISO];
  const long long* dev_bases;  // non-null: [niso][7] bases in device memory (see k_fe_plan)
};

// Bases of isovalue q: the launch arguments, or device memory written by a
// plan kernel ([niso][7]: id x, y, z, output row x, y, z, triangle row).
__device__ __forceinline__ long long base_id(const FeEmitArgs& A, int q, int s) {
  return A.dev_bases ? __ldcg(A.dev_bases + q * 7 + s) : A.pt_id_base[q][s];
}
__device__ __forceinline__ long long base_out(const FeEmitArgs& A, int q, int s) {
  return A.dev_bases ? __ldcg(A.dev_bases + q * 7 + 3 + s) : A.pt_out_base[q][s];
}
__device__ __forceinline__ long long base_tri(const FeEmitArgs& A, int q) {
  return A.dev_bases ? __ldcg(A.dev_bases + q * 7 + 6) : A.tri_out_base[q];
}

// An emit write that would land outside the caller's buffers is skipped and
// recorded in the workspace error word (read by tkmc_fe_check).
__device__ __forceinline__ void record_overflow(long long* info) {
  atomicExch((unsigned long long*)(info + 10), (unsigned long long)TKMC_ERR_CAPACITY);
}

// Device-planned bases whose global point total does not fit int32 ids are
// negative (k_fe_plan_body).  The emit then writes nothing: lane 0 of each
// warp records TKMC_ERR_OVERFLOW (unless an earlier error is recorded) and
// the caller skips its work.  Host-given bases are never negative.
__device__ __forceinline__ bool ids_overflow(long long id_base, long long* info) {
  if (id_base >= 0) return false;
  if ((threadIdx.x & 31) == 0)
    atomicCAS((unsigned long long*)(info + 10), 0ull, (unsigned long long)TKMC_ERR_OVERFLOW);
  return true;
}

// Segmented (width S) inclusive scan.
__device__ __forceinline__ unsigned seg_scan(unsigned x, int sl, int S) {
  for (int o = 1; o < S; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, x, o, S);
    if (sl >= o) x += y;
  }
  return x;
}

// Word record layout in shared memory (32-bit words; odd stride).
//   0-7   crossing masks of the 8 edge groups: x(a) y(a) z(a) x(b) x(c) x(d) y(c) z(b)
//   8     cells with triangles (before the mask)
//   9-16  bit words a a1 b b1 c c1 d d1 (x1 = next node)
//   17-32 int64 id offset of each group's first crossing in this word (lo, hi)
//   33-34 (unused)
//   35-36 j, k of the row
//   37-38 exclusive prefix over the warp's words of points / active cells
constexpr int kRec = 39;
constexpr int kRecMasks = 0, kRecAct = 8, kRecBits = 9, kRecOff = 17, kRecJ = 35, kRecK = 36,
              kRecPB = 37, kRecCB = 38;


__device__ __forceinline__ long long rec_i64(const uint32_t* rec, int at) {
  return (long long)(((unsigned long long)rec[at + 1] << 32) | rec[at]);
}
__device__ __forceinline__ void rec_put_i64(uint32_t* rec, int at, long long v) {
  rec[at] = (uint32_t)(unsigned long long)v;
  rec[at + 1] = (uint32_t)((unsigned long long)v >> 32);
}


// Largest word u of the warp whose record field `field` (non-decreasing in u)
// is <= e.
__device__ __forceinline__ int find_word(const uint32_t* recs, int field, unsigned e) {
  int lo = 0;
#pragma unroll
  for (int step = 16; step >= 1; step >>= 1) {
    const int m = lo + step;
    if (m < 32 && recs[m * kRec + field] <= e) lo = m;
  }
  return lo;
}

__global__ void __launch_bounds__(kThreads, 3)
k_fe_emit_rows(FeDims d, FeWsAll ws, FeEmitArgs A) {
  __shared__ uint64_t s_case[256];
  __shared__ uint32_t s_rec[kThreads / 32][32 * kRec];
  __shared__ long long s_tri[kThreads / 32][32];  // running triangle offset per row segment
  const int isoi = blockIdx.y;
  const FeIsoWs W = iso_ws(ws, isoi);
  const float* __restrict__ vol = block_vol(ws, A.v);
  const int32_t* __restrict__ msk = block_mask(ws, A.mask);
  const float* gm = block_geom(ws, A.geom);
  const int bq = (int)blockIdx.z * (int)gridDim.y + isoi;  // bases of this block and isovalue
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  s_case[tid] = c_case_tris[tid];
  __syncthreads();
  uint32_t* recs = s_rec[warp];
  long long* tri_cur = s_tri[warp];

  const int S = d.S3, logS = d.logS3, G = 32 >> logS;
  const int seg = lane >> logS, sl = lane & (S - 1);
  const int64_t L = d.L, plane = d.L * d.M;
  const uint32_t M32 = (uint32_t)d.M;
  const int64_t n_active = *((volatile long long*)(W.info + 8));
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + tid) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const float iso = A.iso.v[isoi];
  const float x0 = gm[0], y0 = gm[1], z0 = gm[2];
  const float hx = gm[3], hy = gm[4], hz = gm[5];
  const long long idB[3] = {base_id(A, bq, 0), base_id(A, bq, 1), base_id(A, bq, 2)};
  const long long shiftX = base_out(A, bq, 0) - idB[0];
  const long long shiftY = base_out(A, bq, 1) - idB[1];
  const long long shiftZ = base_out(A, bq, 2) - idB[2];
  const long long outT = base_tri(A, bq);
  if (ids_overflow(idB[0], W.info)) return;

  for (int64_t grp = gw; grp * G < n_active; grp += nw) {
    // ---------------- phase 1: lane = (row segment, word) ----------------
    const int64_t item = grp * G + seg;
    const bool valid = item < n_active;
    const int64_t r = valid ? (int64_t)W.work[item] : 0;
    const uint32_t j = (uint32_t)r % M32, k = (uint32_t)r / M32;
    const bool hasY = valid && (j + 1 < M32);
    const bool hasZ = valid && ((int64_t)k + 1 < d.N);
    const bool hasC = hasY && hasZ;
    const int64_t rowbit = r * L;
    long long off[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    long long ota = 0;
    if (valid) {
      const longlong2* ra = reinterpret_cast<const longlong2*>(W.rowoff + r * 4);
      const longlong2 p0 = ra[0], p1 = ra[1];
      off[0] = p0.x + idB[0];
      off[1] = p0.y + idB[1];
      off[2] = p1.x + idB[2];
      ota = p1.y;
    }
    if (hasY) {
      off[3] = W.rowoff[(r + 1) * 4 + 0] + idB[0];
      off[7] = W.rowoff[(r + 1) * 4 + 2] + idB[2];
    }
    if (hasZ) {
      off[4] = W.rowoff[(r + d.M) * 4 + 0] + idB[0];
      off[6] = W.rowoff[(r + d.M) * 4 + 1] + idB[1];
    }
    if (hasC) off[5] = W.rowoff[(r + d.M + 1) * 4 + 0] + idB[0];
    if (sl == 0) tri_cur[seg] = ota;

    for (int w0 = 0; w0 < d.W; w0 += S) {
      const int w = w0 + sl;
      Quad q;
      load_quad(q, W.bits, d, S, rowbit, w, sl, valid, hasY, hasZ);
      const uint32_t xm = low_mask((int)min(L - 1 - 32 * (int64_t)w, (int64_t)32));
      uint32_t m[8];
      m[0] = (q.a ^ shr1(q.a, q.an)) & xm;
      m[1] = hasY ? (q.a ^ q.b) : 0u;
      m[2] = hasZ ? (q.a ^ q.c) : 0u;
      m[3] = (q.b ^ shr1(q.b, q.bn)) & xm;
      m[4] = (q.c ^ shr1(q.c, q.cn)) & xm;
      m[5] = (q.d ^ shr1(q.d, q.dn)) & xm;
      m[6] = hasC ? (q.c ^ q.d) : 0u;
      m[7] = hasC ? (q.b ^ q.d) : 0u;
      const uint32_t act = hasC ? active_cells(q, xm) : 0u;
      // Per-row exclusive prefixes of the eight crossing counts, two per scan.
      unsigned pk[4], ex[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        pk[t] = __popc(m[2 * t]) | (__popc(m[2 * t + 1]) << 16);
        const unsigned inc = seg_scan(pk[t], sl, S);
        ex[t] = inc - pk[t];
        pk[t] = __shfl_sync(0xffffffffu, inc, S - 1, S);  // segment total
      }
      // Warp-wide prefixes of this row's points and active cells per word:
      // the work lists of phase 2.
      const unsigned np = __popc(m[0]) + __popc(m[1]) + __popc(m[2]);
      const unsigned nc = __popc(act);
      unsigned wl = np | (nc << 16);
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, wl, o);
        if (lane >= o) wl += y;
      }
      const unsigned wtot = __shfl_sync(0xffffffffu, wl, 31);
      const unsigned NP = wtot & 0xffffu, NC = wtot >> 16;
      wl -= np | (nc << 16);
      uint32_t* rec = recs + lane * kRec;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        rec[kRecMasks + g] = m[g];
        const unsigned e = (g & 1) ? (ex[g >> 1] >> 16) : (ex[g >> 1] & 0xffffu);
        rec_put_i64(rec, kRecOff + 2 * g, off[g] + e);
      }
      rec[kRecAct] = act;
      rec[kRecBits + 0] = q.a; rec[kRecBits + 1] = shr1(q.a, q.an);
      rec[kRecBits + 2] = q.b; rec[kRecBits + 3] = shr1(q.b, q.bn);
      rec[kRecBits + 4] = q.c; rec[kRecBits + 5] = shr1(q.c, q.cn);
      rec[kRecBits + 6] = q.d; rec[kRecBits + 7] = shr1(q.d, q.dn);
      rec[kRecJ] = j;
      rec[kRecK] = k;
      rec[kRecPB] = wl & 0xffffu;
      rec[kRecCB] = wl >> 16;
#pragma unroll
      for (int g = 0; g < 8; ++g) {  // carry the row totals into the next chunk
        const unsigned t = (g & 1) ? (pk[g >> 1] >> 16) : (pk[g >> 1] & 0xffffu);
        off[g] += t;
      }
      __syncwarp();

      // ---------------- phase 2a: points, lane = one crossing ----------------
      for (unsigned e0 = 0; e0 < NP; e0 += 32) {
        const unsigned e = e0 + lane;
        if (e < NP) {
          const int u = find_word(recs, kRecPB, e);
          const uint32_t* R = recs + u * kRec;
          int kk = (int)(e - R[kRecPB]);
          const uint32_t m0 = R[0], m1 = R[1], m2 = R[2];
          const int c0 = __popc(m0), c1 = __popc(m1);
          int type;
          uint32_t mm;
          if (kk < c0) {
            type = 0; mm = m0;
          } else if (kk < c0 + c1) {
            type = 1; mm = m1; kk -= c0;
          } else {
            type = 2; mm = m2; kk -= c0 + c1;
          }
          const int bit = nth_set_bit(mm, kk);
          const uint32_t uj = R[kRecJ], uk = R[kRecK];
          const int64_t n = 32 * (int64_t)(w0 + (u & (S - 1))) + bit;
          const int64_t node = ((int64_t)uk * d.M + uj) * L + n;
          const int64_t step = type == 0 ? 1 : (type == 1 ? L : plane);
          const float s0 = __ldg(vol + node), s1 = __ldg(vol + node + step);
          const long long shift = type == 0 ? shiftX : (type == 1 ? shiftY : shiftZ);
          const long long row = rec_i64(R, kRecOff + 2 * type) +
                                __popc(mm & ((1u << bit) - 1u)) + shift;
          if (row < 0 || row >= A.points_cap) {
            record_overflow(W.info);
          } else {
            const float t = interp_t(iso, s0, s1);
            const float px = coord(x0, n, hx);
            const float py = coord(y0, uj, hy);
            const float pz = coord(z0, (int64_t)uk + A.k_offset, hz);
            const float px1 = type == 0 ? coord(x0, n + 1, hx) : px;
            const float py1 = type == 1 ? coord(y0, (int64_t)uj + 1, hy) : py;
            const float pz1 = type == 2 ? coord(z0, (int64_t)uk + 1 + A.k_offset, hz) : pz;
            float* o = A.points + row * 3;
            o[0] = lerp_ref(px, px1, t);
            o[1] = lerp_ref(py, py1, t);
            o[2] = lerp_ref(pz, pz1, t);
          }
        }
      }

      // ---------------- phase 2b: triangles, lane = one active cell ----------------
      for (unsigned e0 = 0; e0 < NC; e0 += 32) {
        const unsigned e = e0 + lane;
        const bool ve = e < NC;
        int useg = -1;
        unsigned nt = 0;
        uint64_t pkc = 0;
        const uint32_t* R = recs;
        int cb = 0;
        int64_t n = 0;
        if (ve) {
          const int u = find_word(recs, kRecCB, e);
          R = recs + u * kRec;
          useg = u >> logS;
          cb = nth_set_bit(R[kRecAct], (int)(e - R[kRecCB]));
          n = 32 * (int64_t)(w0 + (u & (S - 1))) + cb;
          const int cs = cell_case(cb, R[kRecBits + 0], R[kRecBits + 1], R[kRecBits + 2],
                                   R[kRecBits + 3], R[kRecBits + 4], R[kRecBits + 5],
                                   R[kRecBits + 6], R[kRecBits + 7]);
          pkc = s_case[cs];
          nt = (unsigned)(pkc >> 60);
          if (nt && msk) {
            const int64_t cell = ((int64_t)R[kRecK] * d.ny + R[kRecJ]) * d.nx + n;
            if (__ldg(msk + cell) != 0) nt = 0;
          }
        }
        // Exclusive scan of nt within each run of lanes of one row.
        unsigned incl = nt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const int prev_seg = __shfl_up_sync(0xffffffffu, useg, 1);
        const bool head = lane == 0 || prev_seg != useg;
        const uint32_t hm = __ballot_sync(0xffffffffu, head);
        const int first = 31 - __clz(hm & (lane == 31 ? 0xffffffffu : ((2u << lane) - 1u)));
        const unsigned before_run = __shfl_sync(0xffffffffu, incl, first > 0 ? first - 1 : 0);
        const unsigned base_excl = first > 0 ? before_run : 0u;
        const long long tbase = ve ? tri_cur[useg] : 0;
        const bool last = lane == 31 || ((hm >> (lane + 1)) & 1u);
        if (nt) {
          const long long tpos = outT + tbase + (long long)(incl - nt - base_excl);
          if (tpos < 0 || tpos + nt > A.conn_cap) {
            record_overflow(W.info);
          } else {
            const uint32_t below = (1u << cb) - 1u;
            const uint32_t below1 = cb == 31 ? 0xffffffffu : ((2u << cb) - 1u);
            int32_t* o = A.conn + tpos * 3;
            for (unsigned t = 0; t < 3 * nt; ++t) {
              const unsigned ed = (unsigned)(pkc >> (4 * t)) & 0xfu;
              const unsigned gp = (unsigned)(kEdgeGroup >> (4 * ed)) & 0xfu;
              const unsigned g = gp & 7u;
              const uint32_t lim = (gp & 8u) ? below1 : below;
              o[t] = (int32_t)(rec_i64(R, kRecOff + 2 * g) + __popc(R[kRecMasks + g] & lim));
            }
          }
        }
        __syncwarp();
        if (ve && last) tri_cur[useg] = tbase + (long long)(incl - base_excl);
        __syncwarp();
      }
      __syncwarp();
    }
  }
}

// ------------------------------------------------------------------------
// K3 (words): emit with work proportional to the active words
// ------------------------------------------------------------------------
//
// A warp takes up to 32 active rows at a time.  For each row, the union of
// the word-activity masks of the four node rows around it (row, +y, +z,
// +y+z) marks every word where any of its eight point-id sequences or its
// triangle sequence advances; all other words contribute nothing.  Those
// words ("units") of all 32 rows are packed into batches of 32 lanes:
//   1. lane = unit: load the unit's four bit words, form the crossing masks
//      and the unit's triangle count, and scan them per row (segmented) into
//      absolute offsets;
//   2. lane = one crossing of the batch: emit the point;
//   3. lane = one active cell of the batch: emit its triangles.

constexpr int kMaxAW = 8;  // rows up to 8192 nodes take this kernel

// Unit record (32-bit words, odd stride).
constexpr int kUR = 39;
constexpr int kURMask = 0;   // 8 crossing masks
constexpr int kURAct = 8;    // cells with triangles
constexpr int kURBits = 9;   // a a1 b b1 c c1 d d1
constexpr int kUROff = 17;   // 8 x int64 id offsets at the unit's first node
constexpr int kURTri = 33;   // int64 triangle offset of the unit's first cell
constexpr int kURSlot = 35;  // row slot in the warp
constexpr int kURW = 36;     // word index in the row
constexpr int kURPB = 37;    // exclusive prefix of points over the batch
constexpr int kURCB = 38;    // exclusive prefix of active cells over the batch
// Row slot record (32-bit words).
constexpr int kSR = 21;
constexpr int kSROff = 0;    // 8 x int64 running id offsets
constexpr int kSRTri = 16;   // int64 running triangle offset
constexpr int kSRJ = 18, kSRK = 19, kSRUB = 20;  // j, k, first unit of the row

struct EmitSmem {
  uint32_t unit[kThreads / 32][32 * kUR];
  uint32_t slot[kThreads / 32][32 * kSR + 1];
  uint32_t umask[kThreads / 32][32 * kMaxAW];
};

// Position of the k-th set bit across the AW words of m (k < total popcount).
__device__ __forceinline__ int nth_set_bit_multi(const uint32_t* m, int AW, int k) {
  for (int i = 0; i < AW; ++i) {
    const int c = __popc(m[i]);
    if (k < c) return 32 * i + nth_set_bit(m[i], k);
    k -= c;
  }
  return -1;
}

// Largest slot s with rec[s * stride + field] <= e (field non-decreasing).
__device__ __forceinline__ int find_slot(const uint32_t* base, int stride, int field,
                                         unsigned e) {
  int lo = 0;
#pragma unroll
  for (int step = 16; step >= 1; step >>= 1) {
    const int m = lo + step;
    if (m < 32 && base[m * stride + field] <= e) lo = m;
  }
  return lo;
}

__device__ __forceinline__ long long ld_i64(const uint32_t* p) {
  return (long long)(((unsigned long long)p[1] << 32) | p[0]);
}
__device__ __forceinline__ void st_i64(uint32_t* p, long long v) {
  p[0] = (uint32_t)(unsigned long long)v;
  p[1] = (uint32_t)((unsigned long long)v >> 32);
}

// Word w of a row (first node at flat bit rowbit) and bit 0 of word w + 1.
__device__ __forceinline__ uint32_t row_word_next(const uint32_t* __restrict__ bits,
                                                  int64_t rowbit, int w, int64_t L,
                                                  uint32_t* next0) {
  const int64_t rem = L - 32 * (int64_t)w;
  if (rem <= 0) {
    *next0 = 0u;
    return 0u;
  }
  const int64_t pos = rowbit + 32 * (int64_t)w;
  const int64_t q = pos >> 5;
  const int sh = (int)(pos & 31);
  const uint32_t lo = __ldg(bits + q), hi = __ldg(bits + q + 1);
  uint32_t x = sh ? __funnelshift_r(lo, hi, sh) : lo;
  uint32_t nx0 = 0u;
  if (rem > 32) nx0 = sh ? (hi >> sh) & 1u : (hi & 1u);
  *next0 = nx0;
  if (rem < 32) x &= (1u << rem) - 1u;
  return x;
}

__global__ void __launch_bounds__(kThreads, 3)
k_fe_emit_words(FeDims d, FeWsAll ws, FeEmitArgs A) {
  extern __shared__ uint32_t k3_smem[];
  __shared__ uint64_t s_case[256];
  EmitSmem& S = *reinterpret_cast<EmitSmem*>(k3_smem);
  const int isoi = blockIdx.y;
  const FeIsoWs W = iso_ws(ws, isoi);
  const float* __restrict__ vol = block_vol(ws, A.v);
  const int32_t* __restrict__ msk = block_mask(ws, A.mask);
  const float* gm = block_geom(ws, A.geom);
  const int bq = (int)blockIdx.z * (int)gridDim.y + isoi;  // bases of this block and isovalue
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  s_case[tid] = c_case_tris[tid];
  __syncthreads();
  uint32_t* U = S.unit[warp];
  uint32_t* SL = S.slot[warp];
  uint32_t* UM = S.umask[warp];
  const int AW = d.AW;
  const int64_t L = d.L, plane = d.L * d.M;
  const uint32_t M32 = (uint32_t)d.M;
  const int64_t n_active = *((volatile long long*)(W.info + 8));
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + tid) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const float iso = A.iso.v[isoi];
  const float x0 = gm[0], y0 = gm[1], z0 = gm[2];
  const float hx = gm[3], hy = gm[4], hz = gm[5];
  const long long idX = base_id(A, bq, 0), idY = base_id(A, bq, 1),
                  idZ = base_id(A, bq, 2);
  const long long shiftX = base_out(A, bq, 0) - idX;
  const long long shiftY = base_out(A, bq, 1) - idY;
  const long long shiftZ = base_out(A, bq, 2) - idZ;
  const long long outT = base_tri(A, bq);
  if (ids_overflow(idX, W.info)) return;

  for (int64_t grp = gw; grp * 32 < n_active; grp += nw) {
    // ---- rows: lane = one active row ----
    const int64_t item = grp * 32 + lane;
    const bool valid = item < n_active;
    const int64_t r = valid ? (int64_t)W.work[item] : 0;
    const uint32_t j = (uint32_t)r % M32, k = (uint32_t)r / M32;
    const bool hasY = valid && (j + 1 < M32);
    const bool hasZ = valid && ((int64_t)k + 1 < d.N);
    const bool hasC = hasY && hasZ;
    long long off[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    long long ota = 0;
    unsigned nu = 0;
    uint32_t* um = UM + lane * kMaxAW;
    for (int i = 0; i < AW; ++i) {
      uint32_t m = 0;
      if (valid) m = __ldg(W.wact + r * AW + i);
      if (hasY) m |= __ldg(W.wact + (r + 1) * AW + i);
      if (hasZ) m |= __ldg(W.wact + (r + d.M) * AW + i);
      if (hasC) m |= __ldg(W.wact + (r + d.M + 1) * AW + i);
      um[i] = m;
      nu += __popc(m);
    }
    if (valid) {
      const longlong2* ra = reinterpret_cast<const longlong2*>(W.rowoff + r * 4);
      const longlong2 p0 = ra[0], p1 = ra[1];
      off[0] = p0.x + idX;
      off[1] = p0.y + idY;
      off[2] = p1.x + idZ;
      ota = p1.y;
    }
    if (hasY) {
      off[3] = W.rowoff[(r + 1) * 4 + 0] + idX;
      off[7] = W.rowoff[(r + 1) * 4 + 2] + idZ;
    }
    if (hasZ) {
      off[4] = W.rowoff[(r + d.M) * 4 + 0] + idX;
      off[6] = W.rowoff[(r + d.M) * 4 + 1] + idY;
    }
    if (hasC) off[5] = W.rowoff[(r + d.M + 1) * 4 + 0] + idX;
    uint32_t* sl = SL + lane * kSR;
#pragma unroll
    for (int g = 0; g < 8; ++g) st_i64(sl + kSROff + 2 * g, off[g]);
    st_i64(sl + kSRTri, ota);
    sl[kSRJ] = j;
    sl[kSRK] = k;
    unsigned ub = nu;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, ub, o);
      if (lane >= o) ub += y;
    }
    const unsigned NU = __shfl_sync(0xffffffffu, ub, 31);
    sl[kSRUB] = ub - nu;
    __syncwarp();

    for (unsigned u0 = 0; u0 < NU; u0 += 32) {
      // ---- units: lane = one active word ----
      const unsigned e = u0 + lane;
      const bool ve = e < NU;
      int slot = 31, w = 0;
      uint32_t m[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      uint32_t act = 0, qa = 0, qa1 = 0, qb = 0, qb1 = 0, qc = 0, qc1 = 0, qd = 0, qd1 = 0;
      unsigned ntu = 0;
      uint32_t sj = 0, sk = 0;
      if (ve) {
        slot = find_slot(SL, kSR, kSRUB, e);
        const uint32_t* sr = SL + slot * kSR;
        w = nth_set_bit_multi(UM + slot * kMaxAW, AW, (int)(e - sr[kSRUB]));
        sj = sr[kSRJ];
        sk = sr[kSRK];
        const int64_t rr = (int64_t)sk * d.M + sj;
        const int64_t rowbit = rr * L;
        const bool hy = sj + 1 < M32, hz = (int64_t)sk + 1 < d.N, hc = hy && hz;
        uint32_t an, bn = 0, cn = 0, dn = 0;
        qa = row_word_next(W.bits, rowbit, w, L, &an);
        if (hy) qb = row_word_next(W.bits, rowbit + L, w, L, &bn);
        if (hz) qc = row_word_next(W.bits, rowbit + plane, w, L, &cn);
        if (hc) qd = row_word_next(W.bits, rowbit + plane + L, w, L, &dn);
        const uint32_t xm = low_mask((int)min(L - 1 - 32 * (int64_t)w, (int64_t)32));
        qa1 = (qa >> 1) | (an << 31);
        qb1 = (qb >> 1) | (bn << 31);
        qc1 = (qc >> 1) | (cn << 31);
        qd1 = (qd >> 1) | (dn << 31);
        m[0] = (qa ^ qa1) & xm;
        m[1] = hy ? (qa ^ qb) : 0u;
        m[2] = hz ? (qa ^ qc) : 0u;
        m[3] = (qb ^ qb1) & xm;
        m[4] = (qc ^ qc1) & xm;
        m[5] = (qd ^ qd1) & xm;
        m[6] = hc ? (qc ^ qd) : 0u;
        m[7] = hc ? (qb ^ qd) : 0u;
        if (hc) {
          const uint32_t u = (qa ^ qb) | (qa ^ qc) | (qa ^ qd);
          const uint32_t un = (an ^ bn) | (an ^ cn) | (an ^ dn);
          act = (u | (u >> 1) | (un << 31) | (qa ^ qa1)) & xm;
          ntu = tri_count_word(qa, qa1, qb, qb1, qc, qc1, qd, qd1, xm);
          if (msk && act) {
            const int64_t cell0 = ((int64_t)sk * d.ny + sj) * d.nx + 32 * (int64_t)w;
            uint32_t t = act;
            while (t) {
              const int bit = __ffs(t) - 1;
              t &= t - 1;
              if (__ldg(msk + cell0 + bit) != 0) {
                ntu -= (unsigned)(s_case[cell_case(bit, qa, qa1, qb, qb1, qc, qc1, qd, qd1)] >> 60);
                act &= ~(1u << bit);
              }
            }
          }
        }
      }
      // Per-row (segmented) prefixes of the eight crossing counts and the
      // triangle count, carried across batches through the row slot.
      const int key = ve ? slot : -1;
      unsigned ex[5], tot[5];
      bool last = false;
#pragma unroll
      for (int t = 0; t < 4; ++t)
        ex[t] = seg_excl(__popc(m[2 * t]) | (__popc(m[2 * t + 1]) << 16), key, &tot[t], &last);
      ex[4] = seg_excl(ntu, key, &tot[4], &last);
      uint32_t* rec = U + lane * kUR;
      uint32_t* sr = SL + slot * kSR;
      if (ve) {
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          rec[kURMask + g] = m[g];
          const unsigned ee = (g & 1) ? (ex[g >> 1] >> 16) : (ex[g >> 1] & 0xffffu);
          st_i64(rec + kUROff + 2 * g, ld_i64(sr + kSROff + 2 * g) + ee);
        }
        st_i64(rec + kURTri, ld_i64(sr + kSRTri) + ex[4]);
        rec[kURAct] = act;
        rec[kURBits + 0] = qa; rec[kURBits + 1] = qa1;
        rec[kURBits + 2] = qb; rec[kURBits + 3] = qb1;
        rec[kURBits + 4] = qc; rec[kURBits + 5] = qc1;
        rec[kURBits + 6] = qd; rec[kURBits + 7] = qd1;
        rec[kURSlot] = (uint32_t)slot;
        rec[kURW] = (uint32_t)w;
      }
      __syncwarp();
      if (ve && last) {  // advance the row's running offsets past this batch
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          const unsigned tt = (g & 1) ? (tot[g >> 1] >> 16) : (tot[g >> 1] & 0xffffu);
          st_i64(sr + kSROff + 2 * g, ld_i64(sr + kSROff + 2 * g) + tt);
        }
        st_i64(sr + kSRTri, ld_i64(sr + kSRTri) + tot[4]);
      }
      // Batch-wide work lists: points of the unit's own row, active cells.
      const unsigned np = __popc(m[0]) + __popc(m[1]) + __popc(m[2]);
      const unsigned nc = __popc(act);
      unsigned wl = np | (nc << 16);
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, wl, o);
        if (lane >= o) wl += y;
      }
      const unsigned wtot = __shfl_sync(0xffffffffu, wl, 31);
      const unsigned NP = wtot & 0xffffu, NC = wtot >> 16;
      wl -= np | (nc << 16);
      rec[kURPB] = ve ? (wl & 0xffffu) : 0xffffffffu;
      rec[kURCB] = ve ? (wl >> 16) : 0xffffffffu;
      __syncwarp();

      // ---- points: lane = one crossing ----
      for (unsigned p0 = 0; p0 < NP; p0 += 32) {
        const unsigned pe = p0 + lane;
        if (pe < NP) {
          const int u = find_slot(U, kUR, kURPB, pe);
          const uint32_t* R = U + u * kUR;
          int kk = (int)(pe - R[kURPB]);
          const uint32_t m0 = R[0], m1 = R[1], m2 = R[2];
          const int c0 = __popc(m0), c1 = __popc(m1);
          int type;
          uint32_t mm;
          if (kk < c0) {
            type = 0; mm = m0;
          } else if (kk < c0 + c1) {
            type = 1; mm = m1; kk -= c0;
          } else {
            type = 2; mm = m2; kk -= c0 + c1;
          }
          const int bit = nth_set_bit(mm, kk);
          const uint32_t* sr2 = SL + R[kURSlot] * kSR;
          const uint32_t uj = sr2[kSRJ], uk = sr2[kSRK];
          const int64_t n = 32 * (int64_t)R[kURW] + bit;
          const int64_t node = ((int64_t)uk * d.M + uj) * L + n;
          const int64_t step = type == 0 ? 1 : (type == 1 ? L : plane);
          const float s0 = __ldg(vol + node), s1 = __ldg(vol + node + step);
          const long long shift = type == 0 ? shiftX : (type == 1 ? shiftY : shiftZ);
          const long long row = ld_i64(R + kUROff + 2 * type) + __popc(mm & ((1u << bit) - 1u)) +
                                shift;
          if (row < 0 || row >= A.points_cap) {
            record_overflow(W.info);
          } else {
            const float t = interp_t(iso, s0, s1);
            const float px = coord(x0, n, hx);
            const float py = coord(y0, uj, hy);
            const float pz = coord(z0, (int64_t)uk + A.k_offset, hz);
            const float px1 = type == 0 ? coord(x0, n + 1, hx) : px;
            const float py1 = type == 1 ? coord(y0, (int64_t)uj + 1, hy) : py;
            const float pz1 = type == 2 ? coord(z0, (int64_t)uk + 1 + A.k_offset, hz) : pz;
            float* o = A.points + row * 3;
            o[0] = lerp_ref(px, px1, t);
            o[1] = lerp_ref(py, py1, t);
            o[2] = lerp_ref(pz, pz1, t);
          }
        }
      }

      // ---- triangles: lane = one active cell ----
      for (unsigned c0 = 0; c0 < NC; c0 += 32) {
        const unsigned ce = c0 + lane;
        const bool vc = ce < NC;
        int u = -1, cb = 0;
        unsigned nt = 0;
        uint64_t pkc = 0;
        if (vc) {
          u = find_slot(U, kUR, kURCB, ce);
          const uint32_t* R = U + u * kUR;
          cb = nth_set_bit(R[kURAct], (int)(ce - R[kURCB]));
          const int cs = cell_case(cb, R[kURBits + 0], R[kURBits + 1], R[kURBits + 2],
                                   R[kURBits + 3], R[kURBits + 4], R[kURBits + 5],
                                   R[kURBits + 6], R[kURBits + 7]);
          pkc = s_case[cs];
          nt = (unsigned)(pkc >> 60);
        }
        unsigned tt;
        bool lst;
        const unsigned ex_in_unit = seg_excl(nt, u, &tt, &lst);
        // Cells of one unit may span batches: continue from the unit's
        // running triangle offset, then advance it.
        const uint32_t* R = U + (vc ? u : 0) * kUR;
        const long long tb = vc ? ld_i64(R + kURTri) : 0;
        if (nt) {
          const long long tpos = outT + tb + ex_in_unit;
          if (tpos < 0 || tpos + nt > A.conn_cap) {
            record_overflow(W.info);
          } else {
            const uint32_t below = (1u << cb) - 1u;
            const uint32_t below1 = cb == 31 ? 0xffffffffu : ((2u << cb) - 1u);
            int32_t* o = A.conn + tpos * 3;
            for (unsigned t = 0; t < 3 * nt; ++t) {
              const unsigned ed = (unsigned)(pkc >> (4 * t)) & 0xfu;
              const unsigned gp = (unsigned)(kEdgeGroup >> (4 * ed)) & 0xfu;
              const unsigned g = gp & 7u;
              const uint32_t lim = (gp & 8u) ? below1 : below;
              o[t] = (int32_t)(ld_i64(R + kUROff + 2 * g) + __popc(R[kURMask + g] & lim));
            }
          }
        }
        __syncwarp();
        if (vc && lst) st_i64(U + u * kUR + kURTri, tb + tt);
        __syncwarp();
      }
      __syncwarp();
    }
  }
}

// ------------------------------------------------------------------------
// K3 for word-aligned rows: units, then points, then triangles, 32 at a time
// ------------------------------------------------------------------------
//
// A unit is one word of an own node row with output (see K2a-K2c).  A warp
// takes 32 consecutive units.  Lane = unit: load the unit, the four rows'
// bit words, the eight crossing masks around its cells, and the offsets of
// the eight edge groups: the unit's own x/y/z offsets and those of the first
// unit at or after word w of rows b, c and d (the unit order makes that the
// offset of word w's first crossing there).  Then lane = point over all the
// units' own crossings (two volume reads each, the reference's arithmetic),
// and lane = cell over all their cut cells (case from the bits, triangle
// slots by a prefix over the task's cut cells -- consecutive units'
// triangles are consecutive in conn -- ids = group offset + rank of the
// crossing in its word).

// Index of the first unit of node row `row` at word >= w.
__device__ __forceinline__ int64_t unit_at(const FeIsoWs& W, const FeDims& d, int64_t row, int w) {
  int64_t u = __ldg(W.ufirst + row);
  const uint32_t* act = W.wact + row * d.AW;
  const int gw = w >> 5;
  for (int i = 0; i < gw; ++i) u += __popc(__ldg(act + i));
  return u + __popc(__ldg(act + gw) & ((1u << (w & 31)) - 1u));
}

// Shared record of one unit (32-bit words).
constexpr int kUB = 0;     // 8 id offsets of the edge groups (id base included)
constexpr int kUM = 8;     // 8 crossing masks
constexpr int kUQ = 16;    // bit words a a1 b b1 c c1 d d1
constexpr int kUAct = 24;  // cut cells of the word
constexpr int kURow = 25, kUW = 26;  // node row, word
constexpr int kUPP = 27;   // exclusive prefix of points over the warp's units
constexpr int kUPC = 28;   // exclusive prefix of cut cells
constexpr int kUCrd = 29;  // f32 bits of y(j), y(j+1), z(k), z(k+1)
constexpr int kUS = 33;

__device__ __forceinline__ int find_rec(const uint32_t* recs, int field, unsigned e) {
  int lo = 0;
#pragma unroll
  for (int step = 16; step >= 1; step >>= 1)
    if (recs[(lo + step) * kUS + field] <= e) lo += step;
  return lo;
}

__global__ void __launch_bounds__(kThreads, 4)
k_fe_emit_units(FeDims d, FeWsAll ws, FeEmitArgs A) {
  __shared__ uint64_t s_case[256];
  __shared__ uint32_t s_rec[kThreads / 32][32 * kUS];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  griddep_launch();
  s_case[tid] = c_case_groups[tid];  // kThreads == 256
  griddep_wait();  // units, bit words and bases of the passes before
  __syncthreads();
  // blockIdx.y = isovalue; the launch sizes each isovalue's grid row to one
  // wave of resident blocks, whose warps take that isovalue's tasks.
  const int isoi = blockIdx.y;
  const int wq = (int)(((int64_t)blockIdx.x * blockDim.x + tid) >> 5);
  const int nwq = (int)(((int64_t)gridDim.x * blockDim.x) >> 5);
  const FeIsoWs W = iso_ws(ws, isoi);
  const float* __restrict__ vol = block_vol(ws, A.v);
  const int32_t* __restrict__ msk = block_mask(ws, A.mask);
  const float* gm = block_geom(ws, A.geom);
  const int bq = (int)blockIdx.z * (int)gridDim.y + isoi;  // bases of this block and isovalue
  const long long n_own = *((volatile long long*)(W.info + 12));
  uint32_t* U = s_rec[warp];
  const int Wd = d.W, Li = (int)d.L;
  const int64_t L = d.L, plane = d.L * d.M;
  const uint32_t M32 = (uint32_t)d.M;
  const float iso = A.iso.v[isoi];
  const float x0 = gm[0], y0 = gm[1], z0 = gm[2];
  const float hx = gm[3], hy = gm[4], hz = gm[5];
  const long long idX = base_id(A, bq, 0), idY = base_id(A, bq, 1),
                  idZ = base_id(A, bq, 2);
  const long long shX = base_out(A, bq, 0) - idX, shY = base_out(A, bq, 1) - idY,
                  shZ = base_out(A, bq, 2) - idZ;
  const long long outT = base_tri(A, bq);
  // Units per warp task: 32 when the units make at least two such tasks per
  // warp, else 16 -- with few tasks the longest one, not their number, sets
  // the kernel's time (the small slabs of 8 GPUs).
  const int G = n_own > 64 * (long long)nwq ? 32 : 16;
  // A warp's first task is its own index; every later one comes from a
  // counter in the workspace (info[13], tasks taken past the first nwq): a
  // warp that finishes early takes the next task, so the load balances, and
  // the warps in flight work on neighbouring units (the volume rows they
  // read are still in L2).  The index of a warp's next task is fetched while
  // the current one runs.  The last warp of the launch to finish (counted in
  // info[14]) sets both counters back to zero for the next launch; the count
  // pass zeroes them too.
  unsigned long long* next_task = reinterpret_cast<unsigned long long*>(W.info + 13);
  unsigned long long* done_warps = reinterpret_cast<unsigned long long*>(W.info + 14);
  long long grp = wq;
  const bool overflow = ids_overflow(idX, W.info);
  while (!overflow && grp * G < n_own) {
    long long nxt = 0;
    if (lane == 0) nxt = (long long)nwq + (long long)atomicAdd(next_task, 1ull);
    // ---- lane = unit ----
    const int64_t u = lane < G ? grp * G + lane : n_own;
    unsigned np = 0, nc = 0;
    long long task_tri = 0;  // lane 0: the task's first triangle row
    uint32_t* rec = U + lane * kUS;
    if (u < n_own) {
      const uint4* up = reinterpret_cast<const uint4*>(W.units + u);
      const uint4 u0 = __ldg(up), u1 = __ldg(up + 1);
      const int64_t r = u0.x;
      const int w = (int)u0.y;
      const RowQuad q = row_quad(d, r);
      const WordQuad x = load_word_quad(W.bits, q, w, Wd);
      const uint32_t xm = low_mask(Li - 1 - 32 * w);
      const uint32_t a1 = (x.a >> 1) | (x.an << 31), b1 = (x.b >> 1) | (x.bn << 31);
      const uint32_t c1 = (x.c >> 1) | (x.cn << 31), d1 = (x.d >> 1) | (x.dn << 31);
      const uint32_t m0 = (x.a ^ a1) & xm, m1 = x.a ^ x.b, m2 = x.a ^ x.c;
      uint32_t act = 0;
      uint32_t bx = 0, bz = 0, cx = 0, cy = 0, dx = 0;
      if (q.hasC) {
        const uint32_t uu = m1 | m2 | (x.a ^ x.d);
        const uint32_t un = (x.an ^ x.bn) | (x.an ^ x.cn) | (x.an ^ x.dn);
        act = (uu | (uu >> 1) | (un << 31) | m0) & xm;
        if (act) {
          const uint4* pb = reinterpret_cast<const uint4*>(W.units + unit_at(W, d, r + 1, w));
          const uint4* pc = reinterpret_cast<const uint4*>(W.units + unit_at(W, d, r + d.M, w));
          const uint4* pd =
              reinterpret_cast<const uint4*>(W.units + unit_at(W, d, r + d.M + 1, w));
          const uint4 b0 = __ldg(pb), b1r = __ldg(pb + 1), c0 = __ldg(pc), d0 = __ldg(pd);
          bx = b0.z;
          bz = b1r.x;
          cx = c0.z;
          cy = c0.w;
          dx = d0.z;
        }
      }
      rec[kUB + 0] = (uint32_t)(idX + u0.z);
      rec[kUB + 1] = (uint32_t)(idY + u0.w);
      rec[kUB + 2] = (uint32_t)(idZ + u1.x);
      rec[kUB + 3] = (uint32_t)(idX + bx);
      rec[kUB + 4] = (uint32_t)(idX + cx);
      rec[kUB + 5] = (uint32_t)(idX + dx);
      rec[kUB + 6] = (uint32_t)(idY + cy);
      rec[kUB + 7] = (uint32_t)(idZ + bz);
      rec[kUM + 0] = m0;
      rec[kUM + 1] = m1;
      rec[kUM + 2] = m2;
      rec[kUM + 3] = (x.b ^ b1) & xm;
      rec[kUM + 4] = (x.c ^ c1) & xm;
      rec[kUM + 5] = (x.d ^ d1) & xm;
      rec[kUM + 6] = x.c ^ x.d;
      rec[kUM + 7] = x.b ^ x.d;
      rec[kUQ + 0] = x.a; rec[kUQ + 1] = a1;
      rec[kUQ + 2] = x.b; rec[kUQ + 3] = b1;
      rec[kUQ + 4] = x.c; rec[kUQ + 5] = c1;
      rec[kUQ + 6] = x.d; rec[kUQ + 7] = d1;
      rec[kUAct] = act;
      rec[kURow] = (uint32_t)r;
      rec[kUW] = (uint32_t)w;
      rec[kUCrd + 0] = __float_as_uint(coord(y0, q.j, hy));
      rec[kUCrd + 1] = __float_as_uint(coord(y0, (int64_t)q.j + 1, hy));
      rec[kUCrd + 2] = __float_as_uint(coord(z0, (int64_t)q.k + A.k_offset, hz));
      rec[kUCrd + 3] = __float_as_uint(coord(z0, (int64_t)q.k + 1 + A.k_offset, hz));
      task_tri = outT + (long long)(((unsigned long long)u1.w << 32) | u1.z);
      np = __popc(m0) + __popc(m1) + __popc(m2);
      nc = __popc(act);
    }
    unsigned pc = np | (nc << 16);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, pc, o);
      if (lane >= o) pc += y;
    }
    const unsigned tot = __shfl_sync(0xffffffffu, pc, 31);
    pc -= np | (nc << 16);
    // Lanes past the last unit get prefixes no item reaches.
    rec[kUPP] = u < n_own ? (pc & 0xffffu) : 0xffffffffu;
    rec[kUPC] = u < n_own ? (pc >> 16) : 0xffffffffu;
    const unsigned NP = tot & 0xffffu, NC = tot >> 16;
    __syncwarp();

    // ---- lane = point ----
    for (unsigned p0 = 0; p0 < NP; p0 += 32) {
      const unsigned pe = p0 + lane;
      if (pe < NP) {
        const uint32_t* R = U + find_rec(U, kUPP, pe) * kUS;
        int kk = (int)(pe - R[kUPP]);
        const uint32_t mx = R[kUM + 0], my = R[kUM + 1];
        const int cxn = __popc(mx), cyn = __popc(my);
        int type;
        uint32_t mm;
        if (kk < cxn) {
          type = 0; mm = mx;
        } else if (kk < cxn + cyn) {
          type = 1; mm = my; kk -= cxn;
        } else {
          type = 2; mm = R[kUM + 2]; kk -= cxn + cyn;
        }
        const int bit = nth_set_bit(mm, kk);
        const int64_t n = 32 * (int64_t)R[kUW] + bit;
        const int64_t node = (int64_t)R[kURow] * L + n;
        const int64_t step = type == 0 ? 1 : (type == 1 ? L : plane);
        const float s0 = __ldg(vol + node), s1 = __ldg(vol + node + step);
        const long long row = (long long)R[kUB + type] + kk +
                              (type == 0 ? shX : (type == 1 ? shY : shZ));
        if (row < 0 || row >= A.points_cap) {
          record_overflow(W.info);
        } else {
          const float t = interp_t(iso, s0, s1);
          const float px = coord(x0, n, hx);
          const float py = __uint_as_float(R[kUCrd + 0]);
          const float pz = __uint_as_float(R[kUCrd + 2]);
          const float px1 = type == 0 ? coord(x0, n + 1, hx) : px;
          const float py1 = type == 1 ? __uint_as_float(R[kUCrd + 1]) : py;
          const float pz1 = type == 2 ? __uint_as_float(R[kUCrd + 3]) : pz;
          float* o = A.points + row * 3;
          o[0] = lerp_ref(px, px1, t);
          o[1] = lerp_ref(py, py1, t);
          o[2] = lerp_ref(pz, pz1, t);
        }
      }
    }

    // ---- lane = cut cell ----
    long long tcarry = __shfl_sync(0xffffffffu, task_tri, 0);
    for (unsigned c0 = 0; c0 < NC; c0 += 32) {
      const unsigned ce = c0 + lane;
      const bool vc = ce < NC;
      int ui = -1, cb = 0;
      unsigned nt = 0;
      uint64_t pkc = 0;
      if (vc) {
        ui = find_rec(U, kUPC, ce);
        const uint32_t* R = U + ui * kUS;
        cb = nth_set_bit(R[kUAct], (int)(ce - R[kUPC]));
        bool masked = false;
        if (msk) {
          const int64_t r = R[kURow];
          const uint32_t j = (uint32_t)r % M32, k = (uint32_t)r / M32;
          masked = __ldg(msk + ((int64_t)k * d.ny + j) * d.nx + 32 * (int64_t)R[kUW] + cb) != 0;
        }
        if (!masked) {
          pkc = s_case[cell_case(cb, R[kUQ + 0], R[kUQ + 1], R[kUQ + 2], R[kUQ + 3], R[kUQ + 4],
                                 R[kUQ + 5], R[kUQ + 6], R[kUQ + 7])];  // groups, not edges
          nt = (unsigned)(pkc >> 60);
        }
      }
      // The triangles of consecutive units are consecutive in conn, so a
      // cell's first triangle is the task's first triangle plus the
      // triangles of every cut cell before it in the task (in unit, then
      // cell order): one warp scan per batch and a running carry.
      unsigned incl = nt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const unsigned batch_tris = __shfl_sync(0xffffffffu, incl, 31);
      if (nt) {
        const long long tpos = tcarry + (long long)(incl - nt);
        if (tpos < 0 || tpos + nt > A.conn_cap) {
          record_overflow(W.info);
        } else {
          const uint32_t* R = U + ui * kUS;
          const uint32_t below = (1u << cb) - 1u;
          const uint32_t below1 = cb == 31 ? 0xffffffffu : ((2u << cb) - 1u);
          int32_t* o = A.conn + tpos * 3;
          for (unsigned t = 0; t < 3 * nt; ++t) {
            const unsigned gp = (unsigned)(pkc >> (4 * t)) & 0xfu;
            const unsigned g = gp & 7u;
            const uint32_t lim = (gp & 8u) ? below1 : below;
            o[t] = (int32_t)(R[kUB + g] + __popc(R[kUM + g] & lim));
          }
        }
      }
      tcarry += batch_tris;
    }
    __syncwarp();
    grp = __shfl_sync(0xffffffffu, nxt, 0);
  }
  if (lane == 0) {
    __threadfence();  // this warp's last task fetch is ordered before its count
    if (atomicAdd(done_warps, 1ull) == (unsigned long long)nwq - 1) {
      __threadfence();
      atomicExch(next_task, 0ull);
      atomicExch(done_warps, 0ull);
    }
  }
}

// ------------------------------------------------------------------------
// unmerged triangle soup (26_marching_cubes.py:453-503)
// ------------------------------------------------------------------------
//
// The same triangles as the merged output, in the same order (cell order,
// tri-table order), but every vertex written out on its own, SoA x/y/z, with
// example 26's arithmetic: the cell's bounds x_lo = x0 + float(i)*dx,
// x_hi = x_lo + dx, an edge's corners at x_lo + cx*(x_hi - x_lo), and the
// vertex xa + t*(xb - xa), t = (iso - va)/((vb - va) + 1e-10).  One warp per
// cell row: its triangle offset from the row table, its words with output
// from the row's activity mask, lane = cell within a word, a warp prefix of
// the cells' triangle counts for their slots.
__constant__ int c_edge_corners[24] = {0, 1, 1, 2, 3, 2, 0, 3, 4, 5, 5, 6,
                                       7, 6, 4, 7, 0, 4, 1, 5, 3, 7, 2, 6};
__constant__ float c_corner_xyz[3][8] = {{0, 1, 1, 0, 0, 1, 1, 0},
                                         {0, 0, 1, 1, 0, 0, 1, 1},
                                         {0, 0, 0, 0, 1, 1, 1, 1}};

__global__ void __launch_bounds__(kThreads)
k_fe_emit_soup(FeDims d, FeWsAll ws, FeEmitArgs A, float* __restrict__ ox,
               float* __restrict__ oy, float* __restrict__ oz) {
  __shared__ uint64_t s_case[256];
  const int isoi = blockIdx.y;
  const FeIsoWs& W = ws.iso[isoi];
  const int tid = threadIdx.x, lane = tid & 31;
  s_case[tid] = c_case_tris[tid];  // kThreads == 256
  __syncthreads();
  const int64_t L = d.L, plane = d.L * d.M;
  const float iso = A.iso.v[isoi];
  const float x0 = A.geom[0], y0 = A.geom[1], z0 = A.geom[2];
  const float hx = A.geom[3], hy = A.geom[4], hz = A.geom[5];
  const long long tri0 = base_tri(A, isoi);
  const int64_t ncrows = d.ny * (d.N - 1);  // cell rows of this slab
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + tid) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t cr = gw; cr < ncrows; cr += nw) {
    const int64_t j = cr % d.ny, k = cr / d.ny;
    const int64_t r = k * d.M + j;
    const long long t_begin = __ldcg(W.rowoff + r * 4 + 3);
    if (__ldcg(W.rowoff + (r + 1) * 4 + 3) == t_begin) continue;  // no triangles
    long long tb = tri0 + t_begin;
    const float y_lo = __fadd_rn(y0, __fmul_rn(__ll2float_rn((long long)j), hy));
    const float y_hi = __fadd_rn(y_lo, hy);
    const float z_lo = __fadd_rn(z0, __fmul_rn(__ll2float_rn((long long)(k + A.k_offset)), hz));
    const float z_hi = __fadd_rn(z_lo, hz);
    const int64_t rowbit = r * L;
    for (int g = 0; g < d.AW; ++g) {
      uint32_t act = __ldcg(W.wact + r * d.AW + g);
      while (act) {
        const int w = 32 * g + __ffs(act) - 1;
        act &= act - 1u;
        uint32_t an, bn, cn, dn;
        const uint32_t a = row_word_next(W.bits, rowbit, w, L, &an);
        const uint32_t b = row_word_next(W.bits, rowbit + L, w, L, &bn);
        const uint32_t c = row_word_next(W.bits, rowbit + plane, w, L, &cn);
        const uint32_t dd = row_word_next(W.bits, rowbit + plane + L, w, L, &dn);
        const uint32_t a1 = (a >> 1) | (an << 31), b1 = (b >> 1) | (bn << 31);
        const uint32_t c1 = (c >> 1) | (cn << 31), d1 = (dd >> 1) | (dn << 31);
        const int64_t i = 32 * (int64_t)w + lane;
        uint64_t pkc = 0;
        unsigned nt = 0;
        if (i < d.nx && !(A.mask && __ldg(A.mask + (k * d.ny + j) * d.nx + i) != 0)) {
          pkc = s_case[cell_case(lane, a, a1, b, b1, c, c1, dd, d1)];
          nt = (unsigned)(pkc >> 60);
        }
        unsigned ex = nt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned y = __shfl_up_sync(0xffffffffu, ex, o);
          if (lane >= o) ex += y;
        }
        const unsigned total = __shfl_sync(0xffffffffu, ex, 31);
        ex -= nt;
        if (nt) {
          const long long t0 = tb + ex;
          if (t0 < 0 || t0 + nt > A.conn_cap) {
            record_overflow(W.info);
          } else {
            const int64_t n0 = rowbit + i;
            float v[8];
            v[0] = __ldg(A.v + n0);
            v[1] = __ldg(A.v + n0 + 1);
            v[2] = __ldg(A.v + n0 + L + 1);
            v[3] = __ldg(A.v + n0 + L);
            v[4] = __ldg(A.v + n0 + plane);
            v[5] = __ldg(A.v + n0 + plane + 1);
            v[6] = __ldg(A.v + n0 + plane + L + 1);
            v[7] = __ldg(A.v + n0 + plane + L);
            const float x_lo = __fadd_rn(x0, __fmul_rn(__ll2float_rn((long long)i), hx));
            const float x_hi = __fadd_rn(x_lo, hx);
            const float lo[3] = {x_lo, y_lo, z_lo};
            const float wd[3] = {__fsub_rn(x_hi, x_lo), __fsub_rn(y_hi, y_lo),
                                 __fsub_rn(z_hi, z_lo)};
            float* outs[3] = {ox, oy, oz};
            for (unsigned q = 0; q < 3 * nt; ++q) {
              const int e = (int)((pkc >> (4 * q)) & 0xfu);
              const int ca = c_edge_corners[2 * e], cb = c_edge_corners[2 * e + 1];
              const float va = v[ca], vb = v[cb];
              const float tt = __fdiv_rn(__fsub_rn(iso, va), __fadd_rn(__fsub_rn(vb, va), 1.0e-10f));
              const int64_t slot = (t0 + q / 3) * 3 + q % 3;
#pragma unroll
              for (int ax = 0; ax < 3; ++ax) {
                const float pa = __fadd_rn(lo[ax], __fmul_rn(c_corner_xyz[ax][ca], wd[ax]));
                const float pb = __fadd_rn(lo[ax], __fmul_rn(c_corner_xyz[ax][cb], wd[ax]));
                outs[ax][slot] = __fadd_rn(pa, __fmul_rn(tt, __fsub_rn(pb, pa)));
              }
            }
          }
        }
        tb += total;
      }
    }
  }
}

// ------------------------------------------------------------------------
// device-side planning: output bases without a host round trip
// ------------------------------------------------------------------------
//
// From the per-rank totals c[world][niso][4] = {X, Y, Z, T} (for one volume:
// world = 1 and c = the workspace's own totals), the bases of rank `rank`:
// point ids in the single-volume layout (isovalue-major; per isovalue all
// ranks' x points, then all y, then all z), and rows in the rank-local
// output (isovalue-major; x, y, z sections of this rank).  The same sums as
// the host's slab_bases.
__device__ void k_fe_plan_body(const long long* c, int world, int rank, int niso,
                               int shared_output, long long* bases) {
  long long Pq = 0, Tq = 0, lp = 0, lt = 0;
  for (int q = 0; q < niso; ++q) {
    long long tot[4] = {0, 0, 0, 0}, before[4] = {0, 0, 0, 0}, own[4];
    for (int r = 0; r < world; ++r)
      for (int s = 0; s < 4; ++s) {
        const long long v = c[((int64_t)r * niso + q) * 4 + s];
        tot[s] += v;
        if (r < rank) before[s] += v;
      }
    for (int s = 0; s < 4; ++s) own[s] = c[((int64_t)rank * niso + q) * 4 + s];
    long long* b = bases + q * 7;
    b[0] = Pq + before[0];
    b[1] = Pq + tot[0] + before[1];
    b[2] = Pq + tot[0] + tot[1] + before[2];
    if (shared_output) {  // every part writes into one single-volume output
      b[3] = b[0];
      b[4] = b[1];
      b[5] = b[2];
      b[6] = Tq + before[3];
    } else {
      b[3] = lp;
      b[4] = lp + own[0];
      b[5] = lp + own[0] + own[1];
      b[6] = lt;
    }
    Pq += tot[0] + tot[1] + tot[2];
    Tq += tot[3];
    lp += own[0] + own[1] + own[2];
    lt += own[3];
  }
  // Point ids are int32 in conn: a global point total above INT32_MAX
  // cannot be emitted.  Negative id bases tell every emit kernel to write
  // nothing and record TKMC_ERR_OVERFLOW (read back by tkmc_fe_check).
  if (Pq > 0x7fffffffLL)
    for (int q = 0; q < niso; ++q)
      for (int s = 0; s < 3; ++s) bases[q * 7 + s] = -1;
}

__global__ void k_fe_plan(const long long* __restrict__ c, int world, int rank, int niso,
                          int shared_output, long long* __restrict__ bases) {
  griddep_launch();
  griddep_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0) k_fe_plan_body(c, world, rank, niso, shared_output, bases);
}

// ------------------------------------------------------------------------
// totals exchange over NVLink peer memory (z-slab ranks, one GPU each)
// ------------------------------------------------------------------------
//
// Every rank keeps a `gathered` array [world][niso][4] and a flag per peer in
// its own memory, mapped into every other rank (CUDA IPC).  One warp per
// rank: bump the local epoch, store this rank's totals into slot `rank` of
// every rank's gathered array (stores over NVLink), fence, then release
// flags[rank] = epoch into every rank; wait (bounded by %globaltimer) until
// all flags of the local array reach the epoch, then plan from the local
// gathered array exactly as k_fe_plan does.  A wait that runs out records
// TKMC_ERR_DEVICE_TIMEOUT in the workspace and plans from what is there.
constexpr int kMaxRanks = 32;

struct ExchangePeers {
  long long* gathered[kMaxRanks];            // each rank's gathered array (peer pointers)
  unsigned long long* flags[kMaxRanks];      // each rank's flags (peer pointers)
  unsigned long long* slot_epoch[kMaxRanks]; // each rank's [2][world] epochs of the slots
};

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// This slab's own totals {X, Y, Z, T} of isovalue q from the count pass
// alone (word-aligned rows, right after K2a): the super-tile totals of the
// whole super-tiles of own rows, the tile totals of the rest of the whole
// tiles, and the row counts of the last partial tile.  Called by one warp;
// every lane returns the sums.
__device__ void own_totals_from_counts(const FeDims& d, const FeIsoWs& W, long long (&out)[4]) {
  const int lane = threadIdx.x & 31;
  const int64_t n = d.n_own_rows;
  const int64_t tiles = n / kThreads, supers = tiles / kSuperTiles;
  long long a[4] = {0, 0, 0, 0};
  for (int64_t i = lane; i < supers; i += 32)
#pragma unroll
    for (int t = 0; t < 4; ++t) a[t] += __ldcg(W.super + i * 5 + t);
  for (int64_t i = supers * kSuperTiles + lane; i < tiles; i += 32)
#pragma unroll
    for (int t = 0; t < 4; ++t) a[t] += __ldcg(W.agg + i * 5 + t);
  for (int64_t r = tiles * kThreads + lane; r < n; r += 32) {
    const int4 c = __ldcg(reinterpret_cast<const int4*>(W.cnt) + r);
    a[0] += c.x;
    a[1] += c.y;
    a[2] += c.z;
    a[3] += c.w;
  }
#pragma unroll
  for (int t = 0; t < 4; ++t) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a[t] += __shfl_xor_sync(0xffffffffu, a[t], o);
    out[t] = a[t];
  }
}

// from_counts: this rank's totals come from the count pass's tile totals
// (own_totals_from_counts), so the exchange can run as soon as K2a is done,
// concurrently with K2b on another stream; else from the info words the
// offsets pass (or the row scan) wrote.
__global__ void k_fe_exchange_plan(ExchangePeers peers, unsigned long long* epoch, int world,
                                   int rank, int niso, const long long* __restrict__ own_info,
                                   int from_counts, FeDims d, FeWsAll ws, int shared_output,
                                   long long* __restrict__ bases, long long* err,
                                   int64_t wait_ns) {
  const int lane = threadIdx.x;  // one warp
  __shared__ unsigned long long s_epoch;
  __shared__ long long s_own[TKMC_MAX_ISO][4];
  if (lane == 0) s_epoch = ++(*epoch);
  for (int q = 0; q < niso; ++q) {
    if (from_counts) {
      long long o[4];
      own_totals_from_counts(d, ws.iso[q], o);
      if (lane < 4) s_own[q][lane] = o[lane];
    } else if (lane < 4) {
      s_own[q][lane] = own_info[16 * q + lane];
    }
  }
  __syncwarp();
  const unsigned long long ep = s_epoch;
  // This rank's totals {X, Y, Z, T} per isovalue (info[16 q + 0..3]) into
  // slot `rank` of every rank's gathered array.  The array has two halves,
  // used by odd and even epochs: a rank that finished waiting in epoch e may
  // still be reading half e % 2 when a faster peer writes epoch e + 1, and no
  // peer can reach epoch e + 2 before this rank has published e + 1.
  //
  // The two-half argument holds only while every wait succeeds.  So each
  // slot also carries the epoch its totals belong to (slot_epoch, written
  // before the flag is released): a rank whose wait ran out and that went on
  // to later steps can get two epochs ahead of a slow peer and overwrite the
  // half that peer reads; the peer then sees a slot epoch other than its own
  // and records an error instead of planning from newer totals.  After any
  // such error the exchange's state is not trusted: the engine (its
  // exchange) is created again.
  const int64_t hb = (int64_t)(ep & 1ull);
  const int64_t half = hb * world * niso * 4;
  for (int r = lane; r < world; r += 32) {
    long long* dst = peers.gathered[r] + half + (int64_t)rank * niso * 4;
    for (int q = 0; q < niso; ++q)
      for (int t = 0; t < 4; ++t) dst[4 * q + t] = s_own[q][t];
    peers.slot_epoch[r][hb * world + rank] = ep;
  }
  __threadfence_system();
  __syncwarp();
  for (int r = lane; r < world; r += 32) st_release_sys_u64(peers.flags[r] + rank, ep);
  // Wait for every rank's totals in the local array.
  const unsigned long long* mine = peers.flags[rank];
  bool ok = true;
  for (int r = lane; r < world; r += 32) {
    if (ld_acquire_sys_u64(mine + r) >= ep) continue;
    const uint64_t t0 = global_ns();
    while (ld_acquire_sys_u64(mine + r) < ep) {
      if ((int64_t)(global_ns() - t0) > wait_ns) {
        ok = false;
        break;
      }
      __nanosleep(32);
    }
  }
  // Every slot of the half must hold this epoch's totals.
  for (int r = lane; r < world; r += 32)
    if (ld_acquire_sys_u64(peers.slot_epoch[rank] + hb * world + r) != ep) ok = false;
  if (!__all_sync(0xffffffffu, ok) && lane == 0)
    atomicExch((unsigned long long*)err, (unsigned long long)TKMC_ERR_DEVICE_TIMEOUT);
  __syncwarp();
  if (lane == 0)
    k_fe_plan_body(peers.gathered[rank] + half, world, rank, niso, shared_output, bases);
}


// Zero the per-call state of a workspace (n8 8-byte words) before a count
// pass.  Launched right behind the threshold pass, which writes none of it,
// so it runs beside that pass's last blocks; it completes only after the
// threshold pass has (griddep_wait at the end), so a kernel that waits on it
// also sees the bitmask.
__global__ void k_fe_reset(unsigned long long* __restrict__ p, int64_t n8) {
  griddep_launch();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = 0ull;
  griddep_wait();
}

// This workspace's own totals {X, Y, Z, T} of each isovalue (info words
// 16q + 0..3) to dst[4q + 0..3] (device memory or mapped host memory).
__global__ void k_fe_copy_totals(const long long* __restrict__ info, int niso,
                                 long long* __restrict__ dst) {
  const int i = threadIdx.x;
  griddep_launch();
  griddep_wait();
  if (i < 4 * niso) dst[i] = __ldcg(info + 16 * (i >> 2) + (i & 3));
}

// Forget capacity errors recorded by an emit (device timeouts stay).
__global__ void k_fe_clear_capacity_error(FeWsAll ws, int niso) {
  const int q = threadIdx.x;
  if (q < niso && ws.iso[q].info[10] == TKMC_ERR_CAPACITY) ws.iso[q].info[10] = 0;
}

// ------------------------------------------------------------------------
// vertex normals (compute_normals.py:16-90)
// ------------------------------------------------------------------------
//
// The reference scatters every triangle's area-weighted face normal into its
// three vertices with f32 atomics, whose order -- and so whose rounding --
// changes from run to run.  Here the same face normals (same f32 operation
// order, no contraction) are added as 64-bit fixed point: integer addition
// is associative, so the sums do not depend on the order, and they keep
// about 58 bits below the largest face normal instead of f32's 24.  The
// scale is a power of two from a first pass over the faces: the largest
// |component| times 2^kNormValence must stay below 2^62.
constexpr int kNormValence = 6;  // a vertex may sum up to 64 faces of the largest size

__device__ __forceinline__ void face_normal(const float* __restrict__ p, const int32_t* __restrict__ conn,
                                            int64_t t, int32_t* i0, int32_t* i1, int32_t* i2,
                                            float* nx, float* ny, float* nz) {
  *i0 = __ldg(conn + 3 * t);
  *i1 = __ldg(conn + 3 * t + 1);
  *i2 = __ldg(conn + 3 * t + 2);
  const float v0x = __ldg(p + 3 * (int64_t)*i0), v0y = __ldg(p + 3 * (int64_t)*i0 + 1),
              v0z = __ldg(p + 3 * (int64_t)*i0 + 2);
  const float v1x = __ldg(p + 3 * (int64_t)*i1), v1y = __ldg(p + 3 * (int64_t)*i1 + 1),
              v1z = __ldg(p + 3 * (int64_t)*i1 + 2);
  const float v2x = __ldg(p + 3 * (int64_t)*i2), v2y = __ldg(p + 3 * (int64_t)*i2 + 1),
              v2z = __ldg(p + 3 * (int64_t)*i2 + 2);
  const float e1x = __fsub_rn(v1x, v0x), e1y = __fsub_rn(v1y, v0y), e1z = __fsub_rn(v1z, v0z);
  const float e2x = __fsub_rn(v2x, v0x), e2y = __fsub_rn(v2y, v0y), e2z = __fsub_rn(v2z, v0z);
  *nx = __fsub_rn(__fmul_rn(e1y, e2z), __fmul_rn(e1z, e2y));
  *ny = __fsub_rn(__fmul_rn(e1z, e2x), __fmul_rn(e1x, e2z));
  *nz = __fsub_rn(__fmul_rn(e1x, e2y), __fmul_rn(e1y, e2x));
}

// Pass 1: the largest |face normal component| (f32 bits; non-negative
// floats order like their bits) and a flag for ids out of range.
__global__ void __launch_bounds__(kThreads)
k_normals_max(const float* __restrict__ p, const int32_t* __restrict__ conn, int64_t n_pts,
              int64_t n_tris, unsigned* __restrict__ maxbits, unsigned* __restrict__ bad) {
  float m = 0.f;
  unsigned badid = 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n_tris; t += stride) {
    const int32_t a = __ldg(conn + 3 * t), b = __ldg(conn + 3 * t + 1), c = __ldg(conn + 3 * t + 2);
    if (a < 0 || b < 0 || c < 0 || a >= n_pts || b >= n_pts || c >= n_pts) {
      badid = 1;
      continue;
    }
    int32_t i0, i1, i2;
    float nx, ny, nz;
    face_normal(p, conn, t, &i0, &i1, &i2, &nx, &ny, &nz);
    m = fmaxf(m, fmaxf(fabsf(nx), fmaxf(fabsf(ny), fabsf(nz))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    badid |= __shfl_xor_sync(0xffffffffu, badid, o);
  }
  if ((threadIdx.x & 31) == 0) {
    if (m > 0.f) atomicMax(maxbits, __float_as_uint(m));  // NaN/inf never win a max here
    if (badid) atomicOr(bad, 1u);
  }
}

// Power-of-two scale from the largest component (its f32 exponent).
__device__ __forceinline__ int normals_shift(unsigned maxbits) {
  if (maxbits == 0u || maxbits >= 0x7f800000u) return 0;  // no faces, or inf/NaN: unscaled
  const int e = (int)((maxbits >> 23) & 0xff) - 127;       // max < 2^(e+1)
  return 62 - kNormValence - (e + 1);                      // max * 2^shift < 2^(62-valence)
}

// Pass 2: add each face normal to its three vertices, in fixed point.
// A face normal that is not finite makes its vertices' normals NaN, as the
// reference's f32 sums would (nan[v] flags them).
__global__ void __launch_bounds__(kThreads)
k_normals_accumulate(const float* __restrict__ p, const int32_t* __restrict__ conn,
                     int64_t n_tris, const unsigned* __restrict__ maxbits,
                     unsigned long long* __restrict__ acc, unsigned* __restrict__ nan) {
  const int shift = normals_shift(*maxbits);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n_tris; t += stride) {
    int32_t i0, i1, i2;
    float nx, ny, nz;
    face_normal(p, conn, t, &i0, &i1, &i2, &nx, &ny, &nz);
    if (!isfinite(nx) || !isfinite(ny) || !isfinite(nz)) {
      nan[i0] = 1u;
      nan[i1] = 1u;
      nan[i2] = 1u;
      continue;
    }
    const unsigned long long fx = (unsigned long long)__double2ll_rn(ldexp((double)nx, shift));
    const unsigned long long fy = (unsigned long long)__double2ll_rn(ldexp((double)ny, shift));
    const unsigned long long fz = (unsigned long long)__double2ll_rn(ldexp((double)nz, shift));
    const int32_t ids[3] = {i0, i1, i2};
#pragma unroll
    for (int v = 0; v < 3; ++v) {
      unsigned long long* a = acc + 3 * (int64_t)ids[v];
      atomicAdd(a, fx);
      atomicAdd(a + 1, fy);
      atomicAdd(a + 2, fz);
    }
  }
}

// Pass 3: back to f32 and normalise where the length exceeds 1e-10
// (compute_normals.py:63-76; a shorter vector is left as summed).
__global__ void __launch_bounds__(kThreads)
k_normals_normalize(const unsigned long long* __restrict__ acc, const unsigned* __restrict__ nan,
                    int64_t n_pts, const unsigned* __restrict__ maxbits, float* __restrict__ out) {
  const int shift = normals_shift(*maxbits);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_pts; i += stride) {
    if (nan[i]) {
      out[3 * i] = out[3 * i + 1] = out[3 * i + 2] = __int_as_float(0x7fffffff);
      continue;
    }
    const double x = ldexp((double)(long long)acc[3 * i], -shift);
    const double y = ldexp((double)(long long)acc[3 * i + 1], -shift);
    const double z = ldexp((double)(long long)acc[3 * i + 2], -shift);
    const double len = sqrt(x * x + y * y + z * z);
    float* o = out + 3 * i;
    if (len > 1.0e-10) {
      o[0] = (float)(x / len);
      o[1] = (float)(y / len);
      o[2] = (float)(z / len);
    } else {
      o[0] = (float)x;
      o[1] = (float)y;
      o[2] = (float)z;
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
  size_t k2_smem;   // dynamic shared memory of the count kernel (rows not word-aligned)
  int64_t V, nwords, bits_stride, nchunks, sums_stride;
  int64_t unit_cap;  // units (incl. the sentinel) the workspace holds; 0: rows not word-aligned
  size_t off_units, off_ufirst, off_ucnt, off_wcnt, off_super;
  int64_t super_stride;
  size_t off_bits, off_sums, off_cnt, off_wact, off_tot, off_base, off_rowoff, off_work, off_info, off_flags,
      off_agg, off_incl, total;
  size_t reset_bytes;  // end of the per-call state zeroed before each count
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
  d.AW = (int)((W + 31) / 32);
  int S = 1, logS = 0;
  while (S < d.W && S < 32) { S <<= 1; ++logS; }
  d.S = S;
  d.logS = logS;
  // K2a tile: about 8192 staged words per run, a multiple of 8 segments.
  const int G = 32 >> logS;
  int64_t TR = 8192 / d.W;
  if (TR > 256) TR = 256;
  TR = (TR / (8 * G)) * (8 * G);
  if (TR < 8 * G) TR = 8 * G;
  d.TR = (int)TR;
  d.logP = 0;
  d.ctiles = (d.R + TR - 1) / TR;
  const bool aligned = (d.L & 31) == 0;
  d.ntiles = aligned ? (d.R + kThreads - 1) / kThreads : (d.R + kScanRows - 1) / kScanRows;
  d.S3 = S < 8 ? S : 8;
  d.logS3 = logS < 3 ? logS : 3;
  f.k2_smem = (size_t)(2 * k2_stage_words((int)TR, d.W)) * 4;
  // Rows that are not word-aligned are staged whole in shared memory.
  if ((d.L & 31) != 0 && f.k2_smem > 200 * 1024) return false;  // longer than ~90k nodes
  if (d.R > 0xffffffffLL) return false;  // worklist holds uint32 row ids
  f.V = d.L * d.M * d.N;
  f.nwords = (f.V + 31) / 32;
  f.bits_stride = (int64_t)align_up((size_t)(f.nwords + 8), 64);
  f.nchunks = (f.V + 1023) / 1024;
  f.sums_stride = (int64_t)align_up((size_t)(f.nchunks + 2), 32);
  // Unit list: room for every word of the volume, plus the sentinel.
  f.unit_cap = aligned ? f.nwords + 1 : 0;
  if (f.nwords > 0xffffffffLL) return false;  // unit and row indices are uint32
  size_t o = 0;
  f.off_info = o;   o = align_up(o + (size_t)niso * 16 * 8, 256);
  f.off_flags = o;  o = align_up(o + (size_t)niso * d.ntiles * 4, 256);
  f.super_stride = aligned ? (d.ntiles + kSuperTiles - 1) / kSuperTiles * 5 : 0;
  f.off_super = o;  o = align_up(o + (size_t)niso * f.super_stride * 8, 256);
  f.off_agg = o;    o = align_up(o + (size_t)niso * d.ntiles * 5 * 8, 256);
  f.reset_bytes = o;  // info, flags, super-tile and tile totals start at zero
  f.off_incl = o;   o = align_up(o + (size_t)niso * d.ntiles * 5 * 8, 256);
  f.off_tot = o;    o = align_up(o + (size_t)niso * 4 * 8, 256);
  f.off_base = o;   o = align_up(o + (size_t)niso * 8 * 8, 256);
  f.off_cnt = o;    o = align_up(o + (size_t)niso * d.R * 4 * 4, 256);
  f.off_wact = o;   o = align_up(o + (size_t)niso * d.R * d.AW * 4, 256);
  f.off_rowoff = o; o = align_up(o + (size_t)niso * d.R * 4 * 8, 256);
  f.off_work = o;   o = align_up(o + (size_t)niso * d.R * 4, 256);
  f.off_bits = o;   o = align_up(o + (size_t)niso * f.bits_stride * 4, 256);
  f.off_sums = o;   o = align_up(o + (size_t)niso * f.sums_stride * 8, 256);
  f.off_ufirst = o; o = align_up(o + (aligned ? (size_t)niso * d.R * 4 : 0), 256);
  f.off_ucnt = o;   o = align_up(o + (aligned ? (size_t)niso * d.R * 4 : 0), 256);
  f.off_wcnt = o;   o = align_up(o + (aligned ? (size_t)niso * f.nwords * 4 : 0), 256);
  f.off_units = o;  o = align_up(o + (size_t)niso * f.unit_cap * sizeof(FeUnit), 256);
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
    w.sums = reinterpret_cast<uint2*>(b + f.off_sums) + (size_t)q * f.sums_stride;
    w.rowoff = reinterpret_cast<long long*>(b + f.off_rowoff) + (size_t)q * f.d.R * 4;
    w.cnt = reinterpret_cast<int*>(b + f.off_cnt) + (size_t)q * f.d.R * 4;
    w.wact = reinterpret_cast<uint32_t*>(b + f.off_wact) + (size_t)q * f.d.R * f.d.AW;
    w.tot = reinterpret_cast<long long*>(b + f.off_tot) + (size_t)q * 4;
    w.work = reinterpret_cast<uint32_t*>(b + f.off_work) + (size_t)q * f.d.R;
    w.flags = reinterpret_cast<uint32_t*>(b + f.off_flags) + (size_t)q * f.d.ntiles;
    w.super = reinterpret_cast<long long*>(b + f.off_super) + (size_t)q * f.super_stride;
    w.agg = reinterpret_cast<long long*>(b + f.off_agg) + (size_t)q * f.d.ntiles * 5;
    w.incl = reinterpret_cast<long long*>(b + f.off_incl) + (size_t)q * f.d.ntiles * 5;
    w.ufirst = reinterpret_cast<uint32_t*>(b + f.off_ufirst) + (size_t)q * f.d.R;
    w.units = reinterpret_cast<FeUnit*>(b + f.off_units) + (size_t)q * f.unit_cap;
    w.ucnt = reinterpret_cast<uint32_t*>(b + f.off_ucnt) + (size_t)q * f.d.R;
    w.wcnt = reinterpret_cast<uint32_t*>(b + f.off_wcnt) + (size_t)q * f.nwords;
    w.info = reinterpret_cast<long long*>(b + f.off_info) + (size_t)q * 16;
  }
  return a;
}

// Raise a kernel's dynamic shared memory limit once per device (and size),
// so that launch sequences need no attribute calls (they may be captured
// into CUDA graphs).  The limit only ever grows: the check, the attribute
// call and the cached value change together under one lock, so two host
// threads asking for different sizes cannot leave the attribute below the
// cached value.  The cache is stored after the attribute is set, so a
// thread that reads a large enough value without the lock may launch.
template <typename F>
int ensure_smem(F* kernel, size_t bytes, std::atomic<size_t>* per_device) {
  static std::mutex mu;
  int dev = 0;
  TK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_err(TKMC_ERR_CUDA, "device index %d out of range", dev);
  if (per_device[dev].load() >= bytes) return TKMC_OK;
  std::lock_guard<std::mutex> lock(mu);
  if (per_device[dev].load() >= bytes) return TKMC_OK;
  TK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  per_device[dev].store(bytes);
  return TKMC_OK;
}
std::atomic<size_t> g_smem_count[64];
std::atomic<size_t> g_smem_emit_words[64];

// Launch with programmatic stream serialization: the kernel may start while
// the kernel before it in the stream is still running (it waits for it in
// griddep_wait before reading its results), so its launch and prologue
// overlap the predecessor's last blocks.  Inside stream capture this becomes
// a programmatic edge of the graph.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
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

// ------------------------------------------------------------------------
// scan without allocation: scratch in a static device array
// ------------------------------------------------------------------------
//
// For callers that cannot allocate device memory, tkmc_scan_i32_noalloc
// keeps the scan's tile states in this file-scope array instead of a
// caller-provided workspace.  Every GPU that loads the library holds it
// (about 320 KiB) until the process exits.  The layout is the one
// tkmc_scan_i32 uses for its workspace, sized for the largest accepted n.
constexpr int64_t kNoAllocScanMaxN = (int64_t)1 << 26;  // 67,108,864 values
constexpr int64_t kNoAllocScanTiles = kNoAllocScanMaxN / kScanTile;
constexpr size_t kNoAllocFlagsBytes = ((size_t)kNoAllocScanTiles * 4 + 255) / 256 * 256;
constexpr size_t kNoAllocTileBytes = ((size_t)kNoAllocScanTiles * 8 + 255) / 256 * 256;
constexpr size_t kNoAllocScratchBytes = 256 + kNoAllocFlagsBytes + 2 * kNoAllocTileBytes;

__device__ __align__(256) unsigned char g_noalloc_scan_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scan_scratch on the current device, resolved
// once per device.  In host code the array's name is only a host-side
// stand-in; kernels must be given this address.
int noalloc_scratch_address(void** out) {
  static std::mutex mu;
  static void* cache[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return set_err(TKMC_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_err(TKMC_ERR_INVALID_ARG, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scan_scratch);
    if (e != cudaSuccess || !p)
      return set_err(TKMC_ERR_CUDA, "cudaGetSymbolAddress(scan scratch) failed: %s",
                     cudaGetErrorString(e));
    cache[dev] = p;
  }
  *out = cache[dev];
  return TKMC_OK;
}

// The end of a scan call: read the total and the look-back error word back
// (one synchronisation).  With total == NULL the error word is still read,
// so an expired look-back wait is reported either way, except while the
// stream is being captured into a CUDA graph: nothing can be read then, and
// the call returns after the launch.
int scan_finish(const long long* info, int64_t* total, cudaStream_t st) {
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  TK_CUDA(cudaStreamIsCapturing(st, &cap));
  if (cap != cudaStreamCaptureStatusNone) {
    if (total) return set_err(TKMC_ERR_INVALID_ARG, "scan total cannot be read during stream capture");
    return TKMC_OK;
  }
  long long h[3];
  TK_CUDA(cudaMemcpyAsync(h, info, sizeof(h), cudaMemcpyDeviceToHost, st));
  TK_CUDA(cudaStreamSynchronize(st));
  if (h[2]) return set_err(TKMC_ERR_DEVICE_TIMEOUT, "scan look-back wait expired");
  if (total) *total = h[1];
  return TKMC_OK;
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

size_t tkmc_normals_workspace_bytes(int64_t n_pts) {
  if (n_pts < 0) return 0;
  return 256 + align_up((size_t)n_pts * 3 * sizeof(unsigned long long), 256) +
         align_up((size_t)n_pts * sizeof(unsigned), 256);
}

int tkmc_compute_normals(const float* points, const int32_t* conn, int64_t n_pts, int64_t n_tris,
                         void* ws, size_t ws_bytes, float* normals, void* stream) {
  if (n_pts < 0 || n_tris < 0) return set_err(TKMC_ERR_INVALID_ARG, "negative size");
  if ((n_tris > 0 && (!points || !conn)) || (n_pts > 0 && !normals))
    return set_err(TKMC_ERR_INVALID_ARG, "tkmc_compute_normals: NULL argument");
  int rc = check_ws(ws, ws_bytes, tkmc_normals_workspace_bytes(n_pts));
  if (rc) return rc;
  if (n_pts > INT32_MAX) return set_err(TKMC_ERR_OVERFLOW, "more than INT32_MAX points");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned* maxbits = static_cast<unsigned*>(ws);
  unsigned* bad = maxbits + 1;
  unsigned long long* acc = reinterpret_cast<unsigned long long*>(static_cast<char*>(ws) + 256);
  unsigned* nan = reinterpret_cast<unsigned*>(
      static_cast<char*>(ws) + 256 + align_up((size_t)n_pts * 3 * sizeof(unsigned long long), 256));
  TK_CUDA(cudaMemsetAsync(ws, 0, tkmc_normals_workspace_bytes(n_pts), st));
  if (n_tris > 0) {
    const int g = grid_for(n_tris, kThreads, 8);
    k_normals_max<<<g, kThreads, 0, st>>>(points, conn, n_pts, n_tris, maxbits, bad);
    TK_LAUNCHED();
    unsigned hbad = 0;
    TK_CUDA(cudaMemcpyAsync(&hbad, bad, sizeof(hbad), cudaMemcpyDeviceToHost, st));
    TK_CUDA(cudaStreamSynchronize(st));
    if (hbad) return set_err(TKMC_ERR_INVALID_ARG, "conn holds a point id outside [0, n_pts)");
    k_normals_accumulate<<<g, kThreads, 0, st>>>(points, conn, n_tris, maxbits, acc, nan);
    TK_LAUNCHED();
  }
  if (n_pts > 0) {
    k_normals_normalize<<<grid_for(n_pts, kThreads, 8), kThreads, 0, st>>>(acc, nan, n_pts,
                                                                          maxbits, normals);
    TK_LAUNCHED();
  }
  return TKMC_OK;
}

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
  return scan_finish(info, total, st);
}

int tkmc_scan_i32_noalloc(const int32_t* in, int32_t* out, int64_t n, int inclusive,
                          int64_t* total, void* stream) {
  if (n < 0 || (n > 0 && (!in || !out)))
    return set_err(TKMC_ERR_INVALID_ARG, "tkmc_scan_i32_noalloc: bad arguments");
  if (n > kNoAllocScanMaxN)
    return set_err(TKMC_ERR_INVALID_ARG,
                   "tkmc_scan_i32_noalloc: n = %lld exceeds the static scratch limit of %lld "
                   "values; use tkmc_scan_i32 with a workspace",
                   (long long)n, (long long)kNoAllocScanMaxN);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    if (total) *total = 0;
    return TKMC_OK;
  }
  void* scratch = nullptr;
  int rc = noalloc_scratch_address(&scratch);
  if (rc) return rc;
  const int64_t tiles = (n + kScanTile - 1) / kScanTile;
  char* b = static_cast<char*>(scratch);
  long long* info = reinterpret_cast<long long*>(b);  // 0 counter, 1 total, 2 error
  uint32_t* flags = reinterpret_cast<uint32_t*>(b + 256);
  long long* agg = reinterpret_cast<long long*>(b + 256 + kNoAllocFlagsBytes);
  long long* incl = reinterpret_cast<long long*>(b + 256 + kNoAllocFlagsBytes + kNoAllocTileBytes);
  // The array keeps the previous call's contents: the tile counter, the
  // error word and the tile flags must start at zero.
  TK_CUDA(cudaMemsetAsync(scratch, 0, 256 + align_up((size_t)tiles * 4, 256), st));
  k_scan_i32<<<(unsigned)tiles, kThreads, 0, st>>>(in, out, n, inclusive, flags, agg, incl, info,
                                                   g_wait_ns.load(), -1);
  TK_LAUNCHED();
  return scan_finish(info, total, st);
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
  constexpr int kWarps = kThreads / 32;
  uint32_t* bits0 = v.iso[0].bits;
  uint2* sums0 = v.iso[0].sums;
  const int64_t nfull = f.V / 1024;  // full chunks (any 4-byte alignment)
  if (nfull > 0) {
    if (nfull / 4 > 0x7fffffffLL) return set_err(TKMC_ERR_INVALID_ARG, "volume too large");
    launch_threshold_words(niso, nfull, 1, st, scalar, iso, bits0, f.bits_stride, f.nwords,
                           sums0, f.sums_stride, nchunks, 0, nullptr);
    TK_LAUNCHED();
  }
  if (nfull < nchunks) {  // the ragged last chunk
    const int64_t rest = nchunks - nfull;
    const int64_t gb = (rest + kWarps - 1) / kWarps;
    if (gb > 0x7fffffffLL) return set_err(TKMC_ERR_INVALID_ARG, "volume too large");
    k_fe_threshold_scalar<<<(unsigned)gb, kThreads, 0, st>>>(scalar, f.V, iso, niso, bits0,
                                                             f.bits_stride, f.nwords, sums0,
                                                             f.sums_stride, nfull, 0, nullptr);
    TK_LAUNCHED();
  }
  return TKMC_OK;
}

// parts: 1 = the count pass (word-aligned rows: K2a; other rows: the whole
// count and row scan), 2 = the offsets pass (word-aligned rows: K2b; other
// rows: nothing), 3 = both.
static int fe_scan_impl(int64_t nx, int64_t ny, int64_t nz, int ghost_plane, int niso,
                        const int32_t* mask, void* ws, size_t ws_bytes, int parts,
                        void* stream) {
  FeLayout f;
  if (!fe_layout(nx, ny, nz, ghost_plane, niso, &f))
    return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  int rc = check_ws(ws, ws_bytes, f.total);
  if (rc) return rc;
  FeWsAll v = fe_views(f, ws, niso);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool aligned = (f.d.L & 31) == 0;
  if (!(parts & 1)) {
    if (aligned) {
      TK_CUDA(launch_pdl(k_fe_offsets_units, dim3((unsigned)f.d.ntiles, (unsigned)niso),
                         dim3(kThreads), 0, st, f.d, v, f.unit_cap, 0));
      TK_LAUNCHED();
    }
    return TKMC_OK;
  }
  {  // zero the per-call state (info, tile flags and totals)
    const int64_t n8 = (int64_t)(f.reset_bytes - f.off_info) / 8;
    TK_CUDA(launch_pdl(k_fe_reset, dim3((unsigned)grid_for(n8, kThreads, 2)), dim3(kThreads), 0,
                       st, reinterpret_cast<unsigned long long*>(static_cast<char*>(ws) + f.off_info),
                       n8));
    TK_LAUNCHED();
  }
  const int64_t skip = g_skip_tile.exchange(-1);
  if (aligned) {  // no waits between blocks here: the skip hook does not apply
    const dim3 tiles((unsigned)f.d.ntiles, (unsigned)niso);
    // Grids of at most about two waves of blocks (the small slabs of
    // several GPUs) end when their busiest block does: share each block's
    // candidates among all its warps there.
    if (f.d.ntiles * niso <= (int64_t)sm_count() * 8)
      TK_CUDA(launch_pdl(k_fe_count_words_bal, tiles, dim3(kThreads), 0, st, f.d, v, mask));
    else
      TK_CUDA(launch_pdl(k_fe_count_words, tiles, dim3(kThreads), 0, st, f.d, v, mask));
    TK_LAUNCHED();
    if (parts & 2) {
      TK_CUDA(launch_pdl(k_fe_offsets_units, tiles, dim3(kThreads), 0, st, f.d, v, f.unit_cap, 0));
      TK_LAUNCHED();
    }
    return TKMC_OK;
  }
  if (f.k2_smem > 48 * 1024)
    if ((rc = ensure_smem(k_fe_count, f.k2_smem, g_smem_count))) return rc;
  k_fe_count<<<dim3((unsigned)f.d.ctiles, (unsigned)niso), kThreads, f.k2_smem, st>>>(
      f.d, v, mask, f.nwords);
  TK_LAUNCHED();
  k_fe_scan_rows<<<dim3((unsigned)f.d.ntiles, (unsigned)niso), kThreads, 0, st>>>(
      f.d, v, g_wait_ns.load(), skip);
  TK_LAUNCHED();
  return TKMC_OK;
}

int tkmc_fe_scan(int64_t nx, int64_t ny, int64_t nz, int ghost_plane, int niso,
                 const int32_t* mask, void* ws, size_t ws_bytes, void* stream) {
  return fe_scan_impl(nx, ny, nz, ghost_plane, niso, mask, ws, ws_bytes, 3, stream);
}

int tkmc_fe_scan_part(int64_t nx, int64_t ny, int64_t nz, int ghost_plane, int niso,
                      const int32_t* mask, void* ws, size_t ws_bytes, int part, void* stream) {
  if (part != 1 && part != 2)
    return set_err(TKMC_ERR_INVALID_ARG, "tkmc_fe_scan_part: part must be 1 or 2, got %d", part);
  return fe_scan_impl(nx, ny, nz, ghost_plane, niso, mask, ws, ws_bytes, part, stream);
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
  if ((f.d.L & 31) == 0) {  // word-aligned rows keep offsets per unit: fill the row table now
    k_fe_offsets_units<<<dim3((unsigned)f.d.ntiles, (unsigned)niso), kThreads, 0, st>>>(
        f.d, v, f.unit_cap, 1);
    TK_LAUNCHED();
  }
  TK_CUDA(cudaMemcpyAsync(out, v.iso[iso].rowoff, (size_t)f.d.R * 4 * sizeof(long long),
                          cudaMemcpyDeviceToHost, st));
  TK_CUDA(cudaStreamSynchronize(st));
  return TKMC_OK;
}

int tkmc_fe_check(int64_t nx, int64_t ny, int64_t nz, int niso, void* ws, size_t ws_bytes,
                  void* stream) {
  FeLayout f;
  if (!fe_layout(nx, ny, nz, 0, niso, &f)) return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  int rc = check_ws(ws, ws_bytes, f.total);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  long long h[TKMC_MAX_ISO * 16];
  TK_CUDA(cudaMemcpyAsync(h, static_cast<char*>(ws) + f.off_info, (size_t)niso * 16 * 8,
                          cudaMemcpyDeviceToHost, st));
  TK_CUDA(cudaStreamSynchronize(st));
  for (int q = 0; q < niso; ++q) {
    const long long e = h[q * 16 + 10];
    if (e == TKMC_ERR_DEVICE_TIMEOUT)
      return set_err((int)e, "a device wait expired, or a peer was out of step: scan look-back "
                             "or totals exchange (isovalue %d)", q);
    if (e == TKMC_ERR_OVERFLOW)
      return set_err((int)e, "the global point total does not fit int32 point ids: nothing "
                             "was emitted (isovalue %d)", q);
    if (e)
      return set_err((int)e, "fe emit wrote past the output capacity (isovalue %d)", q);
  }
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

static int fe_emit_impl(const float* scalar, int64_t nx, int64_t ny, int64_t nz, int ghost_plane,
                        int64_t k_offset, const float* geom6, const float* isovalues, int niso,
                        const int32_t* mask, void* ws, size_t ws_bytes, const int64_t* pt_id_base,
                        const int64_t* pt_out_base, const int64_t* tri_out_base,
                        const int64_t* bases_dev, float* points, int64_t points_capacity,
                        int32_t* conn, int64_t conn_capacity, void* stream) {
  int rc = check_iso(isovalues, niso);
  if (rc) return rc;
  FeLayout f;
  if (!fe_layout(nx, ny, nz, ghost_plane, niso, &f))
    return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  if ((rc = check_ws(ws, ws_bytes, f.total))) return rc;
  if (!scalar || !geom6 || (!bases_dev && (!pt_id_base || !pt_out_base || !tri_out_base)))
    return set_err(TKMC_ERR_INVALID_ARG, "tkmc_fe_emit: NULL argument");
  FeEmitArgs A{};
  A.dev_bases = reinterpret_cast<const long long*>(bases_dev);
  A.v = scalar;
  A.mask = mask;
  A.points = points;
  A.conn = conn;
  A.points_cap = points ? points_capacity : 0;
  A.conn_cap = conn ? conn_capacity : 0;
  for (int i = 0; i < 6; ++i) A.geom[i] = geom6[i];
  A.k_offset = k_offset;
  for (int q = 0; q < niso; ++q) {
    A.iso.v[q] = isovalues[q];
    if (bases_dev) continue;
    for (int s = 0; s < 3; ++s) {
      A.pt_id_base[q][s] = pt_id_base[3 * q + s];
      A.pt_out_base[q][s] = pt_out_base[3 * q + s];
    }
    A.tri_out_base[q] = tri_out_base[q];
  }
  FeWsAll v = fe_views(f, ws, niso);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (f.d.AW <= kMaxAW) {
    const size_t smem = sizeof(EmitSmem);
    if ((rc = ensure_smem(k_fe_emit_words, smem, g_smem_emit_words))) return rc;
    if (f.unit_cap > 0) {  // word-aligned rows: the unit list; one wave of blocks per isovalue
      TK_CUDA(launch_pdl(k_fe_emit_units, dim3((unsigned)(sm_count() * 4), (unsigned)niso),
                         dim3(kThreads), 0, st, f.d, v, A));
      TK_LAUNCHED();
      return TKMC_OK;
    }
    const int g = grid_for(f.d.n_own_rows, kThreads, 3);
    k_fe_emit_words<<<dim3((unsigned)g, (unsigned)niso), kThreads, smem, st>>>(f.d, v, A);
  } else {
    const int G = 32 >> f.d.logS3;
    const int g = grid_for(f.d.n_own_rows, (kThreads / 32) * G, 8);
    k_fe_emit_rows<<<dim3((unsigned)g, (unsigned)niso), kThreads, 0, st>>>(f.d, v, A);
  }
  TK_LAUNCHED();
  return TKMC_OK;
}

int tkmc_fe_emit(const float* scalar, int64_t nx, int64_t ny, int64_t nz, int ghost_plane,
                 int64_t k_offset, const float* geom6, const float* isovalues, int niso,
                 const int32_t* mask, void* ws, size_t ws_bytes, const int64_t* pt_id_base,
                 const int64_t* pt_out_base, const int64_t* tri_out_base, float* points,
                 int64_t points_capacity, int32_t* conn, int64_t conn_capacity, void* stream) {
  return fe_emit_impl(scalar, nx, ny, nz, ghost_plane, k_offset, geom6, isovalues, niso, mask, ws,
                      ws_bytes, pt_id_base, pt_out_base, tri_out_base, nullptr, points,
                      points_capacity, conn, conn_capacity, stream);
}

int tkmc_fe_emit_dev(const float* scalar, int64_t nx, int64_t ny, int64_t nz, int ghost_plane,
                     int64_t k_offset, const float* geom6, const float* isovalues, int niso,
                     const int32_t* mask, void* ws, size_t ws_bytes, const int64_t* bases_dev,
                     float* points, int64_t points_capacity, int32_t* conn,
                     int64_t conn_capacity, void* stream) {
  if (!bases_dev) return set_err(TKMC_ERR_INVALID_ARG, "tkmc_fe_emit_dev: bases_dev is NULL");
  return fe_emit_impl(scalar, nx, ny, nz, ghost_plane, k_offset, geom6, isovalues, niso, mask, ws,
                      ws_bytes, nullptr, nullptr, nullptr, bases_dev, points, points_capacity,
                      conn, conn_capacity, stream);
}

int tkmc_fe_copy_counts(int64_t nx, int64_t ny, int64_t nz, int niso, const void* ws,
                        size_t ws_bytes, int64_t* dst, void* stream) {
  FeLayout f;
  if (!fe_layout(nx, ny, nz, 0, niso, &f)) return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  int rc = check_ws(const_cast<void*>(ws), ws_bytes, f.total);
  if (rc) return rc;
  if (!dst) return set_err(TKMC_ERR_INVALID_ARG, "dst is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long* info =
      reinterpret_cast<const long long*>(static_cast<const char*>(ws) + f.off_info);
  // This device's memory, or page-locked host memory the device can
  // address: one tiny kernel stores the totals (a copy-engine transfer at
  // the end of a graph-launched step costs several microseconds more).
  // Anything else (pageable host memory, another GPU's memory): a copy.
  cudaPointerAttributes at{};
  int dev = -1;
  if (cudaPointerGetAttributes(&at, dst) == cudaSuccess && cudaGetDevice(&dev) == cudaSuccess &&
      ((at.type == cudaMemoryTypeDevice && at.device == dev) ||
       (at.type == cudaMemoryTypeHost && at.devicePointer != nullptr))) {
    long long* d = static_cast<long long*>(at.type == cudaMemoryTypeHost ? at.devicePointer
                                                                         : static_cast<void*>(dst));
    TK_CUDA(launch_pdl(k_fe_copy_totals, dim3(1), dim3(32), 0, st, info, niso, d));
    TK_LAUNCHED();
    return TKMC_OK;
  }
  cudaGetLastError();  // a pointer the runtime does not know is not an error here
  TK_CUDA(cudaMemcpy2DAsync(dst, 4 * sizeof(long long), info, 16 * sizeof(long long),
                            4 * sizeof(long long), (size_t)niso, cudaMemcpyDefault, st));
  return TKMC_OK;
}

int tkmc_fe_emit_soup(const float* scalar, int64_t nx, int64_t ny, int64_t nz,
                      const float* geom6, const float* isovalues, int niso, const int32_t* mask,
                      void* ws, size_t ws_bytes, const int64_t* tri_out_base, float* out_x,
                      float* out_y, float* out_z, int64_t tri_capacity, void* stream) {
  int rc = check_iso(isovalues, niso);
  if (rc) return rc;
  FeLayout f;
  if (!fe_layout(nx, ny, nz, 0, niso, &f)) return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  if ((rc = check_ws(ws, ws_bytes, f.total))) return rc;
  if (!scalar || !geom6 || !tri_out_base || (tri_capacity > 0 && (!out_x || !out_y || !out_z)))
    return set_err(TKMC_ERR_INVALID_ARG, "tkmc_fe_emit_soup: NULL argument");
  FeEmitArgs A{};
  A.v = scalar;
  A.mask = mask;
  A.conn_cap = tri_capacity;
  for (int i = 0; i < 6; ++i) A.geom[i] = geom6[i];
  for (int q = 0; q < niso; ++q) {
    A.iso.v[q] = isovalues[q];
    A.tri_out_base[q] = tri_out_base[q];
  }
  FeWsAll v = fe_views(f, ws, niso);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((f.d.L & 31) == 0) {  // word-aligned rows keep offsets per unit: fill the row table
    k_fe_offsets_units<<<dim3((unsigned)f.d.ntiles, (unsigned)niso), kThreads, 0, st>>>(
        f.d, v, f.unit_cap, 1);
    TK_LAUNCHED();
  }
  const int64_t ncrows = ny * nz;
  if (ncrows > 0 && nx > 0) {
    k_fe_emit_soup<<<dim3((unsigned)grid_for(ncrows, kThreads / 32, 8), (unsigned)niso), kThreads, 0,
                     st>>>(f.d, v, A, out_x, out_y, out_z);
    TK_LAUNCHED();
  }
  return TKMC_OK;
}

// ---- batches of same-shape blocks ----------------------------------------

size_t tkmc_fe_batch_stride(int64_t nx, int64_t ny, int64_t nz, int niso) {
  return align_up(tkmc_fe_workspace_bytes(nx, ny, nz, niso), 256);
}

static int batch_views(int64_t nx, int64_t ny, int64_t nz, int niso, int64_t nblocks,
                       const float* const* vols, const int32_t* const* masks, void* ws,
                       size_t ws_bytes, FeLayout* f, FeWsAll* v) {
  if (nblocks < 1 || nblocks > 65535)
    return set_err(TKMC_ERR_INVALID_ARG, "nblocks must be in [1, 65535], got %lld",
                   (long long)nblocks);
  if (!fe_layout(nx, ny, nz, 0, niso, f)) return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  if (!vols) return set_err(TKMC_ERR_INVALID_ARG, "vols is NULL");
  const size_t stride = align_up(f->total, 256);
  int rc = check_ws(ws, ws_bytes, stride * (size_t)nblocks);
  if (rc) return rc;
  *v = fe_views(*f, ws, niso);
  v->stride = (int64_t)stride;
  v->vols = vols;
  v->masks = masks;
  return TKMC_OK;
}

int tkmc_fe_count_batch(const float* const* vols, int64_t nblocks, int64_t nx, int64_t ny,
                        int64_t nz, const float* isovalues, int niso, const int32_t* const* masks,
                        void* ws, size_t ws_bytes, int64_t* counts, int64_t* status,
                        void* stream) {
  int rc = check_iso(isovalues, niso);
  if (rc) return rc;
  FeLayout f;
  FeWsAll v;
  if ((rc = batch_views(nx, ny, nz, niso, nblocks, vols, masks, ws, ws_bytes, &f, &v))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  IsoParams iso{};
  for (int t = 0; t < niso; ++t) iso.v[t] = isovalues[t];
  const int64_t nchunks = (f.V + 1023) / 1024, nfull = f.V / 1024;
  const unsigned nb = (unsigned)nblocks;
  // Full chunks by the word kernel, a ragged last chunk by the scalar one.
  if (nfull > 0) {
    launch_threshold_words(niso, nfull, nb, st, nullptr, iso, v.iso[0].bits, f.bits_stride,
                           f.nwords, v.iso[0].sums, f.sums_stride, nchunks, v.stride, vols);
    TK_LAUNCHED();
  }
  if (nfull < nchunks) {
    k_fe_threshold_scalar<<<dim3(1, 1, nb), kThreads, 0, st>>>(
        nullptr, f.V, iso, niso, v.iso[0].bits, f.bits_stride, f.nwords, v.iso[0].sums,
        f.sums_stride, nfull, v.stride, vols);
    TK_LAUNCHED();
  }
  TK_CUDA(cudaMemset2DAsync(static_cast<char*>(ws) + f.off_info, (size_t)v.stride, 0,
                            f.reset_bytes - f.off_info, (size_t)nblocks, st));
  if ((f.d.L & 31) == 0) {
    const dim3 tiles((unsigned)f.d.ntiles, (unsigned)niso, nb);
    k_fe_count_words<<<tiles, kThreads, 0, st>>>(f.d, v, nullptr);
    TK_LAUNCHED();
    k_fe_offsets_units<<<tiles, kThreads, 0, st>>>(f.d, v, f.unit_cap, 0);
    TK_LAUNCHED();
  } else {
    if (f.k2_smem > 48 * 1024)
      if ((rc = ensure_smem(k_fe_count, f.k2_smem, g_smem_count))) return rc;
    k_fe_count<<<dim3((unsigned)f.d.ctiles, (unsigned)niso, nb), kThreads, f.k2_smem, st>>>(
        f.d, v, nullptr, f.nwords);
    TK_LAUNCHED();
    k_fe_scan_rows<<<dim3((unsigned)f.d.ntiles, (unsigned)niso, nb), kThreads, 0, st>>>(
        f.d, v, g_wait_ns.load(), -1);
    TK_LAUNCHED();
  }
  for (int q = 0; q < niso; ++q) {
    const char* info = static_cast<const char*>(ws) + f.off_info + (size_t)q * 16 * 8;
    if (counts)
      TK_CUDA(cudaMemcpy2DAsync(counts + 4 * q, (size_t)niso * 4 * 8, info, (size_t)v.stride, 4 * 8,
                                (size_t)nblocks, cudaMemcpyDefault, st));
    if (status)
      TK_CUDA(cudaMemcpy2DAsync(status + q, (size_t)niso * 8, info + 10 * 8, (size_t)v.stride, 8,
                                (size_t)nblocks, cudaMemcpyDefault, st));
  }
  return TKMC_OK;
}

int tkmc_fe_emit_batch(const float* const* vols, int64_t nblocks, int64_t nx, int64_t ny,
                       int64_t nz, const float* geoms, const float* isovalues, int niso,
                       const int32_t* const* masks, void* ws, size_t ws_bytes,
                       const int64_t* bases, float* points, int64_t points_capacity,
                       int32_t* conn, int64_t conn_capacity, int64_t* status, void* stream) {
  int rc = check_iso(isovalues, niso);
  if (rc) return rc;
  FeLayout f;
  FeWsAll v;
  if ((rc = batch_views(nx, ny, nz, niso, nblocks, vols, masks, ws, ws_bytes, &f, &v))) return rc;
  if (!geoms || !bases) return set_err(TKMC_ERR_INVALID_ARG, "tkmc_fe_emit_batch: NULL argument");
  v.geoms = geoms;
  FeEmitArgs A{};
  A.points = points;
  A.conn = conn;
  A.points_cap = points ? points_capacity : 0;
  A.conn_cap = conn ? conn_capacity : 0;
  A.dev_bases = reinterpret_cast<const long long*>(bases);
  for (int q = 0; q < niso; ++q) A.iso.v[q] = isovalues[q];
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned nb = (unsigned)nblocks;
  const int per_block =
      (int)std::max<int64_t>(1, std::min<int64_t>(64, (int64_t)sm_count() * 8 / nblocks));
  if (f.unit_cap > 0) {
    k_fe_emit_units<<<dim3((unsigned)per_block, (unsigned)niso, nb), kThreads, 0, st>>>(f.d, v, A);
  } else if (f.d.AW <= kMaxAW) {
    const size_t smem = sizeof(EmitSmem);
    if ((rc = ensure_smem(k_fe_emit_words, smem, g_smem_emit_words))) return rc;
    k_fe_emit_words<<<dim3((unsigned)per_block, (unsigned)niso, nb), kThreads, smem, st>>>(f.d, v, A);
  } else {
    k_fe_emit_rows<<<dim3((unsigned)per_block, (unsigned)niso, nb), kThreads, 0, st>>>(f.d, v, A);
  }
  TK_LAUNCHED();
  if (status)
    for (int q = 0; q < niso; ++q)
      TK_CUDA(cudaMemcpy2DAsync(status + q, (size_t)niso * 8,
                                static_cast<const char*>(ws) + f.off_info + (size_t)q * 16 * 8 + 10 * 8,
                                (size_t)v.stride, 8, (size_t)nblocks, cudaMemcpyDefault, st));
  return TKMC_OK;
}

// ---- totals exchange over NVLink peer memory ------------------------------

struct tkmc_exchange_impl {
  int world, rank, niso, device;
  // one allocation: flags [world] u64 | gathered [2][world][niso][4] i64 |
  // slot epochs [2][world] u64 | epoch u64
  char* base;
  size_t off_gathered, off_slot_epoch, off_epoch, bytes;
  ExchangePeers peers;
  void* opened[kMaxRanks];
};

size_t tkmc_exchange_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int tkmc_exchange_create(int world, int rank, int niso, void** out, void* handle) {
  if (!out || !handle) return set_err(TKMC_ERR_INVALID_ARG, "tkmc_exchange_create: NULL argument");
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || niso < 1 ||
      niso > TKMC_MAX_ISO)
    return set_err(TKMC_ERR_INVALID_ARG, "tkmc_exchange_create: bad world/rank/niso");
  tkmc_exchange_impl* x = new tkmc_exchange_impl();
  x->world = world;
  x->rank = rank;
  x->niso = niso;
  cudaError_t e = cudaGetDevice(&x->device);
  x->off_gathered = align_up((size_t)world * 8, 256);
  x->off_slot_epoch = x->off_gathered + align_up((size_t)2 * world * niso * 4 * 8, 256);
  x->off_epoch = x->off_slot_epoch + align_up((size_t)2 * world * 8, 256);
  x->bytes = x->off_epoch + 256;
  if (e == cudaSuccess) e = cudaMalloc(&x->base, x->bytes);
  if (e == cudaSuccess) e = cudaMemset(x->base, 0, x->bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), x->base);
  if (e != cudaSuccess) {
    if (x->base) cudaFree(x->base);
    delete x;
    return set_err(TKMC_ERR_CUDA, "tkmc_exchange_create: %s", cudaGetErrorString(e));
  }
  *out = x;
  return TKMC_OK;
}

int tkmc_exchange_connect(void* xp, const void* handles) {
  tkmc_exchange_impl* x = static_cast<tkmc_exchange_impl*>(xp);
  if (!x || !handles) return set_err(TKMC_ERR_INVALID_ARG, "tkmc_exchange_connect: NULL argument");
  const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int r = 0; r < x->world; ++r) {
    char* b = x->base;
    if (r != x->rank) {
      void* p = nullptr;
      const cudaError_t e = cudaIpcOpenMemHandle(&p, h[r], cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess)
        return set_err(TKMC_ERR_CUDA, "tkmc_exchange_connect: rank %d: %s", r, cudaGetErrorString(e));
      x->opened[r] = p;
      b = static_cast<char*>(p);
    }
    x->peers.flags[r] = reinterpret_cast<unsigned long long*>(b);
    x->peers.gathered[r] = reinterpret_cast<long long*>(b + x->off_gathered);
    x->peers.slot_epoch[r] = reinterpret_cast<unsigned long long*>(b + x->off_slot_epoch);
  }
  return TKMC_OK;
}

int tkmc_exchange_connect_local(void* xp, void* const* members) {
  tkmc_exchange_impl* x = static_cast<tkmc_exchange_impl*>(xp);
  if (!x || !members)
    return set_err(TKMC_ERR_INVALID_ARG, "tkmc_exchange_connect_local: NULL argument");
  for (int r = 0; r < x->world; ++r) {
    const tkmc_exchange_impl* m = static_cast<const tkmc_exchange_impl*>(members[r]);
    if (!m || m->world != x->world || m->rank != r || m->niso != x->niso || m->device != x->device)
      return set_err(TKMC_ERR_INVALID_ARG, "tkmc_exchange_connect_local: member %d does not match", r);
    x->peers.flags[r] = reinterpret_cast<unsigned long long*>(m->base);
    x->peers.gathered[r] = reinterpret_cast<long long*>(m->base + m->off_gathered);
    x->peers.slot_epoch[r] = reinterpret_cast<unsigned long long*>(m->base + m->off_slot_epoch);
  }
  return TKMC_OK;
}

static int exchange_plan_impl(void* xp, int64_t nx, int64_t ny, int64_t nz, int ghost_plane,
                              const void* ws, size_t ws_bytes, int shared_output,
                              int64_t* bases_dev, int after_count_pass, void* stream) {
  tkmc_exchange_impl* x = static_cast<tkmc_exchange_impl*>(xp);
  if (!x || !bases_dev) return set_err(TKMC_ERR_INVALID_ARG, "tkmc_exchange_plan: NULL argument");
  FeLayout f;
  if (!fe_layout(nx, ny, nz, ghost_plane, x->niso, &f))
    return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  int rc = check_ws(const_cast<void*>(ws), ws_bytes, f.total);
  if (rc) return rc;
  const long long* info = reinterpret_cast<const long long*>(static_cast<const char*>(ws) + f.off_info);
  // Word-aligned rows keep tile totals after the count pass; other rows
  // finish their totals in the count pass itself (the row scan).
  const int from_counts = after_count_pass && (f.d.L & 31) == 0;
  k_fe_exchange_plan<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      x->peers, reinterpret_cast<unsigned long long*>(x->base + x->off_epoch), x->world, x->rank,
      x->niso, info, from_counts, f.d, fe_views(f, const_cast<void*>(ws), x->niso), shared_output,
      reinterpret_cast<long long*>(bases_dev), const_cast<long long*>(info) + 10,
      g_wait_ns.load());
  TK_LAUNCHED();
  return TKMC_OK;
}

int tkmc_exchange_plan(void* xp, int64_t nx, int64_t ny, int64_t nz, int ghost_plane,
                       const void* ws, size_t ws_bytes, int shared_output, int64_t* bases_dev,
                       void* stream) {
  return exchange_plan_impl(xp, nx, ny, nz, ghost_plane, ws, ws_bytes, shared_output, bases_dev,
                            0, stream);
}

int tkmc_exchange_plan_counts(void* xp, int64_t nx, int64_t ny, int64_t nz, int ghost_plane,
                              const void* ws, size_t ws_bytes, int shared_output,
                              int64_t* bases_dev, void* stream) {
  return exchange_plan_impl(xp, nx, ny, nz, ghost_plane, ws, ws_bytes, shared_output, bases_dev,
                            1, stream);
}

int tkmc_exchange_destroy(void* xp) {
  tkmc_exchange_impl* x = static_cast<tkmc_exchange_impl*>(xp);
  if (!x) return TKMC_OK;
  for (int r = 0; r < x->world; ++r)
    if (x->opened[r]) cudaIpcCloseMemHandle(x->opened[r]);
  cudaFree(x->base);
  delete x;
  return TKMC_OK;
}

int tkmc_fe_copy_status(int64_t nx, int64_t ny, int64_t nz, int niso, const void* ws,
                        size_t ws_bytes, int64_t* dst, void* stream) {
  FeLayout f;
  if (!fe_layout(nx, ny, nz, 0, niso, &f)) return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  int rc = check_ws(const_cast<void*>(ws), ws_bytes, f.total);
  if (rc) return rc;
  if (!dst) return set_err(TKMC_ERR_INVALID_ARG, "dst is NULL");
  TK_CUDA(cudaMemcpy2DAsync(dst, sizeof(long long),
                            static_cast<const char*>(ws) + f.off_info + 10 * sizeof(long long),
                            16 * sizeof(long long), sizeof(long long), (size_t)niso,
                            cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
  return TKMC_OK;
}

int tkmc_fe_plan(const int64_t* all_counts_dev, int world, int rank, int niso,
                 int shared_output, int64_t* bases_dev, void* stream) {
  if (!all_counts_dev || !bases_dev) return set_err(TKMC_ERR_INVALID_ARG, "tkmc_fe_plan: NULL");
  if (world < 1 || rank < 0 || rank >= world || niso < 1 || niso > TKMC_MAX_ISO)
    return set_err(TKMC_ERR_INVALID_ARG, "tkmc_fe_plan: bad world/rank/niso");
  TK_CUDA(launch_pdl(k_fe_plan, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
                     reinterpret_cast<const long long*>(all_counts_dev), world, rank, niso,
                     shared_output, reinterpret_cast<long long*>(bases_dev)));
  TK_LAUNCHED();
  return TKMC_OK;
}

int tkmc_fe_clear_capacity_error(int64_t nx, int64_t ny, int64_t nz, int niso, void* ws,
                                 size_t ws_bytes, void* stream) {
  FeLayout f;
  if (!fe_layout(nx, ny, nz, 0, niso, &f)) return set_err(TKMC_ERR_INVALID_ARG, "bad grid or niso");
  int rc = check_ws(ws, ws_bytes, f.total);
  if (rc) return rc;
  k_fe_clear_capacity_error<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(fe_views(f, ws, niso),
                                                                            niso);
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
  rc = tkmc_fe_emit(scalar, nx, ny, nz, 0, 0, geom6, isovalues, niso, mask, ws, ws_bytes, id, id,
                    tri, points, points_capacity, conn, conn_capacity, stream);
  if (rc) return rc;
  return tkmc_fe_check(nx, ny, nz, niso, ws, ws_bytes, stream);
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
