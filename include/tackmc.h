/*
 * tackmc.h -- C ABI of libtackmc.so, the sm_100a isosurface library behind
 * tack_b200.algorithms.flying_edges.
 *
 * Every entry point takes plain pointers, 64-bit sizes and a CUDA stream
 * passed as `void*` (NULL = legacy default stream).  Device pointers must
 * belong to the device that is current on the calling thread.  Scratch
 * space is a caller-provided workspace whose size the matching
 * *_workspace_bytes() function returns.  The only entry points that allocate
 * or free device memory are tkmc_exchange_create (one small buffer per rank,
 * shared with the other ranks through CUDA IPC) and tkmc_exchange_destroy,
 * which frees it.
 * Every entry point returns an int status (TKMC_OK == 0); on failure
 * tkmc_last_error() returns a thread-local message.  Nothing exits, traps or
 * waits without a bound.
 *
 * Reference interfaces replaced (paths inside berkgeveci/tack):
 *   packages/tack-vis/src/tack/algorithms/flying_edges.py
 *   packages/tack-core/src/tack/algorithms/scan.py
 *   packages/tack-core/src/tack/runtime/cuda_backend.py
 *   packages/tack-vis/examples/26_marching_cubes.py
 */
#ifndef TACKMC_H
#define TACKMC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define TKMC_OK                  0
#define TKMC_ERR_INVALID_ARG     1  /* bad size, null pointer, misuse          */
#define TKMC_ERR_WORKSPACE       2  /* workspace smaller than required         */
#define TKMC_ERR_OVERFLOW        3  /* point total does not fit int32 ids      */
#define TKMC_ERR_DEVICE_TIMEOUT  4  /* a bounded device-side wait expired      */
#define TKMC_ERR_CUDA            5  /* CUDA runtime error (message has detail) */
#define TKMC_ERR_CAPACITY        6  /* caller's output buffers too small       */

/* Largest number of isovalues one fe call classifies in a single volume read. */
#define TKMC_MAX_ISO 8

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int tkmc_version(void);

/* Thread-local message describing the last failed call on this thread. */
const char* tkmc_last_error(void);

/* Number of kernels this library has launched in this process (all devices).
 * Used by benchmarks to count their own launches inside a timed region. */
uint64_t tkmc_launch_count(void);

/* Host-only: copy the marching-cubes case tables the kernels use into host
 * arrays: tri_table[256*16] (edge ids, -1 padded), num_tris[256],
 * edge_corners[24].  Any pointer may be NULL.
 * Replaces: flying_edges.py:33-306 (_EDGE_CORNERS, _TRI_TABLE, _NUM_TRIS) and
 * flying_edges.py:344-371 (MCTables / _get_tables). */
int tkmc_mc_tables(int32_t* tri_table, int32_t* num_tris, int32_t* edge_corners);

/* ---- field reductions --------------------------------------------------- */

/* Workspace for tkmc_reduce_f32 over n values. */
size_t tkmc_reduce_workspace_bytes(int64_t n);

/* min, max and sum of n f32 values in one read, written to HOST out4 as
 * doubles {min, max, sum, nan_count}.  min/max ignore NaN (CUDA fminf/fmaxf
 * semantics); all-NaN or n == 0 gives min = +inf, max = -inf.  The sum is
 * accumulated in f64 in a fixed order (deterministic for a given device).
 * Synchronises `stream`.
 * Replaces: cuda_backend.py:576-615 (CUDABackend.reduce_field) and the
 * reduce_sum/min/max_f32 kernels at cuda_backend.py:44-106, whose element
 * count is a 32-bit uint (cuda_backend.py:49); n here is 64-bit. */
int tkmc_reduce_f32(const float* values, int64_t n, void* workspace,
                    size_t workspace_bytes, double* out4, void* stream);

/* ---- prefix scan -------------------------------------------------------- */

/* Workspace for tkmc_scan_i32 over n values. */
size_t tkmc_scan_workspace_bytes(int64_t n);

/* Single-pass (decoupled look-back) prefix sum of n int32 values.
 * inclusive == 0: out[i] = sum(in[0..i-1]), out[0] = 0;  inclusive != 0:
 * out[i] = sum(in[0..i]).  Sums are carried in int64 and stored as int32
 * (two's-complement wrap, as the reference's int32 fields do); *total (HOST,
 * may be NULL) receives the exact int64 sum of all n values.  `in` and `out`
 * may alias.  Synchronises `stream` once, to read the total and the look-back
 * error word back, also when total is NULL: an expired look-back wait returns
 * TKMC_ERR_DEVICE_TIMEOUT either way.  While `stream` is being captured into
 * a CUDA graph nothing is read back (total must then be NULL) and no timeout
 * can be reported.
 * Replaces: scan.py:81-102 (exclusive_scan) and scan.py:105-123
 * (inclusive_scan). */
int tkmc_scan_i32(const int32_t* in, int32_t* out, int64_t n, int inclusive,
                  void* workspace, size_t workspace_bytes, int64_t* total,
                  void* stream);

/* tkmc_scan_i32 without any device allocation, for callers that cannot
 * allocate: code called from inside another application's time step (an
 * in-situ hook in a simulation that has reserved the GPU's memory up front,
 * where cudaMalloc can fail or stall the application's other streams by
 * synchronising the device), or hosts whose allocator is owned by another
 * framework.  Same arguments and results as tkmc_scan_i32, minus the
 * workspace.  No counterpart in the reference (its scan allocates fields,
 * scan.py:94-101).
 * Scratch is a static device array inside this library (about 320 KiB,
 * held by every GPU that loads it until the process exits); n is limited to
 * 2^26 = 67,108,864 values and larger n returns TKMC_ERR_INVALID_ARG.  The
 * first call on a device looks up the array's device address (a synchronous
 * runtime call): make that first call before any stream capture.  All calls
 * share the one array: calls that overlap on the GPU (other streams or
 * threads, same device) race, so serialise them. */
int tkmc_scan_i32_noalloc(const int32_t* in, int32_t* out, int64_t n,
                          int inclusive, int64_t* total, void* stream);

/* ---- vertex normals ------------------------------------------------------ */

/* Workspace for tkmc_compute_normals over n_pts points. */
size_t tkmc_normals_workspace_bytes(int64_t n_pts);

/* Smooth vertex normals of a triangle mesh: each triangle's area-weighted
 * face normal cross(v1 - v0, v2 - v0) (f32, the reference's operation order)
 * is added to its three vertices, then every vertex sum longer than 1e-10 is
 * normalised (shorter ones are left as summed).  points f32 [n_pts*3]
 * interleaved, conn int32 [n_tris*3], normals f32 [n_pts*3] out.  The sums
 * are 64-bit fixed point, so the result does not depend on the order of the
 * additions (the reference's f32 atomics do); a vertex of a face whose
 * normal is not finite gets NaN.  Point ids outside [0, n_pts) return
 * TKMC_ERR_INVALID_ARG.  Synchronises `stream` once (the id check).
 * Replaces: compute_normals.py:16-90 (compute_normals). */
int tkmc_compute_normals(const float* points, const int32_t* conn, int64_t n_pts,
                         int64_t n_tris, void* workspace, size_t workspace_bytes,
                         float* normals, void* stream);

/* ---- flying edges (merged-point marching cubes) ------------------------- */
/*
 * Grid: nx, ny, nz cells; (nx+1)*(ny+1)*(nz+1) f32 node values, i fastest,
 * k slowest (flying_edges.py:313-341 UniformGrid).  Cells with mask[cell] != 0
 * emit no triangles (mask is nullable; int32 per cell, flying_edges.py:441-477).
 *
 * ghost_plane != 0 marks node plane nz as a read-only ghost owned by the next
 * z-slab: its nodes close this slab's last cell layer, but its x/y edges are
 * not counted in this slab's totals (they belong to the next slab, whose
 * point-id bases make the ids match).  Single-volume calls pass 0.
 *
 * Output layout is the reference's (flying_edges.py:480-656): all x-edge
 * points in node-row order, then all y-edge points, then all z-edge points;
 * triangles in cell-row order, tri-table order within a cell; points f32
 * [x,y,z] interleaved, conn int32 triples.  For several isovalues each
 * isovalue's block follows the previous one.
 */

/* Workspace for the fe calls on this grid and number of isovalues. */
size_t tkmc_fe_workspace_bytes(int64_t nx, int64_t ny, int64_t nz, int niso);

/* Pass 1 (count): classify every node against each isovalue in ONE read of
 * the volume, count x/y/z edge crossings per node row and triangles per cell
 * row, and scan them into per-row offsets kept in the workspace.  Writes
 * HOST counts[niso*4] = {X, Y, Z, T} per isovalue (this slab's own totals).
 * Synchronises `stream`.
 * Replaces: flying_edges.py:663-715 (_count_block: _fe_count_edges_xyz,
 * _fe_count_rows, to_numpy and numpy cumsum). */
int tkmc_fe_count(const float* scalar, int64_t nx, int64_t ny, int64_t nz,
                  int ghost_plane, const float* isovalues, int niso,
                  const int32_t* mask, void* workspace, size_t workspace_bytes,
                  int64_t* counts, void* stream);

/* Pass 2 (emit): write points and connectivity using the offsets left in the
 * workspace by tkmc_fe_count (same arguments).  Per isovalue q:
 *   pt_id_base[3q+s]  is added to section-s (0=x,1=y,2=z) offsets to form the
 *                     point ids stored in conn;
 *   pt_out_base[3q+s] is added to the same offsets to form the row index in
 *                     `points` where section-s points are written;
 *   tri_out_base[q]   is the row index in `conn` of q's first triangle.
 * For one volume: pt_id_base = pt_out_base = {P0, P0+X, P0+X+Y} with P0 the
 * points of earlier isovalues, tri_out_base = earlier triangles.  geom6 =
 * {x0, y0, z0, dx, dy, dz}; k_offset is the global index of this slab's node
 * plane 0 (point z uses float(k + k_offset), exactly as the reference).
 * points_capacity / conn_capacity are the rows (of 3) the buffers hold; a
 * write beyond them is skipped and recorded, and tkmc_fe_check then returns
 * TKMC_ERR_CAPACITY.  Asynchronous on `stream`.
 * Replaces: flying_edges.py:718-746 (_emit_block: _fe_emit_points_xyz,
 * _fe_emit_tris). */
int tkmc_fe_emit(const float* scalar, int64_t nx, int64_t ny, int64_t nz,
                 int ghost_plane, int64_t k_offset, const float* geom6,
                 const float* isovalues, int niso, const int32_t* mask,
                 void* workspace, size_t workspace_bytes,
                 const int64_t* pt_id_base, const int64_t* pt_out_base,
                 const int64_t* tri_out_base, float* points,
                 int64_t points_capacity, int32_t* conn, int64_t conn_capacity,
                 void* stream);

/* tkmc_fe_emit with the bases in DEVICE memory instead of host arrays:
 * bases_dev[7q .. 7q+6] = {id x, id y, id z, row x, row y, row z, triangle
 * row} of isovalue q, as tkmc_fe_plan writes them.  Nothing is read on the
 * host, so count -> plan -> emit runs without a host round trip (and can be
 * captured in a CUDA graph).  Capacities as in tkmc_fe_emit.  Asynchronous.
 * No counterpart in the reference, whose emit takes host offsets
 * (flying_edges.py:718-746). */
int tkmc_fe_emit_dev(const float* scalar, int64_t nx, int64_t ny, int64_t nz,
                     int ghost_plane, int64_t k_offset, const float* geom6,
                     const float* isovalues, int niso, const int32_t* mask,
                     void* workspace, size_t workspace_bytes,
                     const int64_t* bases_dev, float* points,
                     int64_t points_capacity, int32_t* conn,
                     int64_t conn_capacity, void* stream);

/* Copy the own totals {X, Y, Z, T} per isovalue (niso*4 int64) that the
 * last count left in the workspace to dst (device memory or page-locked
 * host memory; a one-warp kernel stores them when the device can address
 * dst, a copy otherwise).  Asynchronous. */
int tkmc_fe_copy_counts(int64_t nx, int64_t ny, int64_t nz, int niso,
                        const void* workspace, size_t workspace_bytes,
                        int64_t* dst, void* stream);

/* Unmerged triangle soup of the last tkmc_fe_count on this workspace (a
 * single volume, ghost_plane 0): the same triangles in the same order as
 * tkmc_fe_emit's conn, every vertex written out, SoA: out_x/out_y/out_z
 * [3*T] with vertex v of triangle t at 3t+v, positions computed as
 * 26_marching_cubes.py:453-503 (emit_triangles) computes them (cell bounds
 * x_lo = x0 + float(i)*dx, x_hi = x_lo + dx, corner x_lo + cx*(x_hi -
 * x_lo)).  tri_out_base[q] = first triangle row of isovalue q.
 * tri_capacity = triangles the arrays hold; writes beyond are skipped and
 * reported by tkmc_fe_check.  Asynchronous.  No counterpart in the
 * reference library: example 26's classify_cells + exclusive_scan +
 * emit_triangles pipeline. */
int tkmc_fe_emit_soup(const float* scalar, int64_t nx, int64_t ny, int64_t nz,
                      const float* geom6, const float* isovalues, int niso,
                      const int32_t* mask, void* workspace, size_t workspace_bytes,
                      const int64_t* tri_out_base, float* out_x, float* out_y,
                      float* out_z, int64_t tri_capacity, void* stream);

/* ---- batches of same-shape blocks (flying_edges_multiblock) ------------ */
/*
 * Many blocks of one grid shape in one launch per phase instead of a
 * sequence of launches per block (flying_edges.py:766-832 launches count
 * and emit kernels per block, with host round trips).  vols and masks are
 * DEVICE arrays of nblocks device pointers (masks may be NULL, or hold NULL
 * entries); the workspace holds nblocks workspaces of
 * tkmc_fe_batch_stride() bytes; nblocks <= 65535.
 */

/* Bytes per block of a batch workspace (a multiple of 256). */
size_t tkmc_fe_batch_stride(int64_t nx, int64_t ny, int64_t nz, int niso);

/* Count every block: counts[b*niso*4 + 4q + s] = {X, Y, Z, T} and
 * status[b*niso + q] = the device status word (0 or TKMC_ERR_*), both
 * copied to device or page-locked host memory (either may be NULL).
 * Asynchronous. */
int tkmc_fe_count_batch(const float* const* vols, int64_t nblocks, int64_t nx,
                        int64_t ny, int64_t nz, const float* isovalues, int niso,
                        const int32_t* const* masks, void* workspace,
                        size_t workspace_bytes, int64_t* counts, int64_t* status,
                        void* stream);

/* Emit every block after tkmc_fe_count_batch: geoms DEVICE [nblocks][6]
 * {x0, y0, z0, dx, dy, dz}; bases DEVICE [nblocks][niso][7] as
 * tkmc_fe_emit_dev's (ids, output rows, triangle row of each block and
 * isovalue); one shared output; status as in tkmc_fe_count_batch (capacity
 * errors).  Asynchronous. */
int tkmc_fe_emit_batch(const float* const* vols, int64_t nblocks, int64_t nx,
                       int64_t ny, int64_t nz, const float* geoms,
                       const float* isovalues, int niso,
                       const int32_t* const* masks, void* workspace,
                       size_t workspace_bytes, const int64_t* bases,
                       float* points, int64_t points_capacity, int32_t* conn,
                       int64_t conn_capacity, int64_t* status, void* stream);

/* ---- totals exchange over NVLink peer memory ----------------------------- */
/*
 * For z-slab ranks, one GPU and one process each: instead of an NCCL
 * all-gather of the totals followed by tkmc_fe_plan, one kernel stores this
 * rank's totals straight into every rank's memory (CUDA IPC mappings over
 * NVLink), raises a per-call epoch flag in each, waits (bounded; a wait that
 * runs out records TKMC_ERR_DEVICE_TIMEOUT, read by tkmc_fe_check) for every
 * rank's flag, and plans.  Every rank must make the same calls in the same
 * order, on its own GPU.  No counterpart in the reference (it has no
 * multi-GPU path).
 *   create: allocate this rank's exchange buffer; writes its IPC handle
 *           (tkmc_exchange_handle_bytes bytes) for the other ranks.
 *   connect: open every rank's handle (handles in rank order).
 *   plan: after tkmc_fe_scan on this rank's slab; bases_dev as tkmc_fe_plan.
 *         Each slot of the gathered totals carries its epoch; a slot from
 *         another epoch (a peer out of step after an expired wait) records
 *         TKMC_ERR_DEVICE_TIMEOUT as well.  After that error, destroy the
 *         exchange on every rank and create it again.
 *   destroy: after every rank has finished its last plan (a barrier).
 */
size_t tkmc_exchange_handle_bytes(void);
int tkmc_exchange_create(int world, int rank, int niso, void** exchange, void* handle);
int tkmc_exchange_connect(void* exchange, const void* handles);
/* Connect without IPC: `members` are all ranks' exchanges (rank order, this
 * one included), created in this process on this device.  For emulating the
 * group in one process: kernels that wait on one another must not run as
 * separate launches on one GPU, so only one member may call
 * tkmc_exchange_plan -- its wait then ends by the time limit
 * (tkmc_set_wait_limit_ns) with TKMC_ERR_DEVICE_TIMEOUT. */
int tkmc_exchange_connect_local(void* exchange, void* const* members);
int tkmc_exchange_plan(void* exchange, int64_t nx, int64_t ny, int64_t nz,
                       int ghost_plane, const void* workspace, size_t workspace_bytes,
                       int shared_output, int64_t* bases_dev, void* stream);
int tkmc_exchange_destroy(void* exchange);
/* tkmc_exchange_plan right after the count pass (tkmc_fe_scan_part part 1):
 * this rank's totals are summed from the count pass's tile totals, so the
 * exchange -- peer stores, the wait for the slowest rank, the plan -- can
 * run on a second stream while the offsets pass (part 2) runs on the first;
 * the emit then waits for both.  Same arguments and results as
 * tkmc_exchange_plan.  No counterpart in the reference. */
int tkmc_exchange_plan_counts(void* exchange, int64_t nx, int64_t ny, int64_t nz,
                              int ghost_plane, const void* workspace,
                              size_t workspace_bytes, int shared_output,
                              int64_t* bases_dev, void* stream);

/* Copy the device status word of each isovalue (niso int64: 0, or the
 * TKMC_ERR_* code the last count/emit recorded -- TKMC_ERR_DEVICE_TIMEOUT,
 * TKMC_ERR_CAPACITY) to dst (device or page-locked host memory), so that
 * the status of many workspaces can be read with one synchronisation.
 * Asynchronous. */
int tkmc_fe_copy_status(int64_t nx, int64_t ny, int64_t nz, int niso,
                        const void* workspace, size_t workspace_bytes,
                        int64_t* dst, void* stream);

/* Device-side planning: from DEVICE all_counts_dev[world][niso][4] (the
 * totals of every z-slab part, in z order; for one volume world = 1 and the
 * workspace's own totals) write bases_dev[niso*7] for part `rank`: point ids
 * in the single-volume layout, and output rows either in a part-local output
 * (shared_output = 0: the part's x, y, z points then its triangles, per
 * isovalue; the sums of tack_b200.distributed.slab_bases) or in one shared
 * single-volume output (shared_output != 0: rows = ids, triangle rows
 * global).  When the global point total (all ranks and isovalues) exceeds
 * INT32_MAX, the id bases are set negative: the emit kernels then write
 * nothing and record TKMC_ERR_OVERFLOW, which tkmc_fe_check returns.
 * Asynchronous. */
int tkmc_fe_plan(const int64_t* all_counts_dev, int world, int rank, int niso,
                 int shared_output, int64_t* bases_dev, void* stream);

/* Forget TKMC_ERR_CAPACITY recorded by an emit into too-small buffers, so
 * that the emit can be repeated into larger ones (device timeouts stay
 * recorded).  Asynchronous. */
int tkmc_fe_clear_capacity_error(int64_t nx, int64_t ny, int64_t nz, int niso,
                                 void* workspace, size_t workspace_bytes,
                                 void* stream);

/* Synchronise `stream` and report any error the device recorded in the
 * workspace during the last count/emit (TKMC_ERR_DEVICE_TIMEOUT,
 * TKMC_ERR_CAPACITY, TKMC_ERR_OVERFLOW from device-planned bases), else
 * TKMC_OK. */
int tkmc_fe_check(int64_t nx, int64_t ny, int64_t nz, int niso,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Phase entry points of tkmc_fe_count, for callers that time or overlap the
 * phases.  classify = one volume read -> node bitmasks (asynchronous);
 * scan = counts + offsets from the bitmasks (asynchronous);
 * read_counts = copy counts to HOST and check the device error word
 * (synchronises).  classify + scan + read_counts == tkmc_fe_count.
 * scan_part splits scan in two: part 1 = the count pass (the per-row
 * counts and the totals; on rows whose length is a multiple of 32 nodes,
 * only the counts and their tile totals), part 2 = the offsets pass (the
 * per-row offsets and the output units; nothing on other rows).  Part 1
 * then part 2 == scan; between them tkmc_exchange_plan_counts may run on
 * another stream. */
int tkmc_fe_classify(const float* scalar, int64_t nx, int64_t ny, int64_t nz,
                     const float* isovalues, int niso, void* workspace,
                     size_t workspace_bytes, void* stream);
int tkmc_fe_scan(int64_t nx, int64_t ny, int64_t nz, int ghost_plane,
                 int niso, const int32_t* mask, void* workspace,
                 size_t workspace_bytes, void* stream);
int tkmc_fe_scan_part(int64_t nx, int64_t ny, int64_t nz, int ghost_plane,
                      int niso, const int32_t* mask, void* workspace,
                      size_t workspace_bytes, int part, void* stream);
int tkmc_fe_read_counts(int64_t nx, int64_t ny, int64_t nz, int niso,
                        void* workspace, size_t workspace_bytes,
                        int64_t* counts, void* stream);

/* Copy to HOST the per-node-row exclusive offsets of the last
 * tkmc_fe_count / tkmc_fe_scan for isovalue `iso` (for rows of a multiple of
 * 32 nodes, whose count pass keeps offsets per word, the row table is first
 * filled in the workspace from the per-row counts):
 * out[4*r + s], s = 0..3: x, y, z point offsets (each relative to its own
 * section) and triangle offset of node row r = k*(ny+1) + j (the triangle
 * offset of the cell row (j, k) when j < ny and k < nz).  (ny+1)*(nz+1)
 * rows.  Synchronises `stream`.
 * Replaces the xo/yo/zo/tri_offsets arrays of flying_edges.py:693-715
 * (_count_block); those add the x total to yo and x+y totals to zo. */
int tkmc_fe_row_offsets(int64_t nx, int64_t ny, int64_t nz, int niso, int iso,
                        const void* workspace, size_t workspace_bytes,
                        int64_t* out, void* stream);

/* Whole filter for one volume into caller buffers of fixed capacity:
 * count, then emit if points_capacity >= sum of points and conn_capacity >=
 * sum of triangles (capacities in rows of 3).  counts as in tkmc_fe_count.
 * Returns TKMC_ERR_CAPACITY (with counts filled, nothing emitted) when the
 * buffers are too small, so the caller can grow them and call tkmc_fe_emit.
 * Replaces: flying_edges.py:749-763 (flying_edges) for C callers. */
int tkmc_fe_run(const float* scalar, int64_t nx, int64_t ny, int64_t nz,
                const float* geom6, const float* isovalues, int niso,
                const int32_t* mask, void* workspace, size_t workspace_bytes,
                float* points, int64_t points_capacity, int32_t* conn,
                int64_t conn_capacity, int64_t* counts, void* stream);

/* Per-cell marching-cubes classification (the per-cell form of
 * 26_marching_cubes.py:435-450 classify_cells): cases[cell] = 8-corner case
 * index, ntris[cell] = triangles of that case (0 where mask != 0).  Either
 * output may be NULL.  Uses the fe workspace for niso = 1.  Asynchronous. */
int tkmc_mc_classify_cells(const float* scalar, int64_t nx, int64_t ny,
                           int64_t nz, float isovalue, const int32_t* mask,
                           void* workspace, size_t workspace_bytes,
                           uint8_t* cases, int32_t* ntris, void* stream);

/* ---- test hooks --------------------------------------------------------- */

/* Bound, in nanoseconds, on every device-side wait (decoupled look-back).
 * Default 1e9.  Values <= 0 restore the default.  Process-wide. */
void tkmc_set_wait_limit_ns(int64_t ns);

/* Testing: make the next fe scan launch skip publishing the status of tile
 * `tile` (-1 = off) so that its successors' bounded waits expire and the call
 * returns TKMC_ERR_DEVICE_TIMEOUT instead of hanging.  One-shot. */
void tkmc_test_skip_publish(int64_t tile);

#ifdef __cplusplus
}
#endif

#endif /* TACKMC_H */
