/*
 * fe_oracle.c -- CPU restatement of berkgeveci/tack's flying-edges
 * isosurface (tack-vis) and of the core scan/reduction it is checked with.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle: the tests, the
 * smoke check and the benchmark's CPU-baseline leg call it as the checker or
 * as the timed CPU baseline.  The product (tack_b200 + libtackmc.so) never
 * links, loads or calls it.
 *
 * Each function restates one reference kernel loop for loop, with the same
 * float arithmetic: f32 values, f32 isovalue, f32 grid scalars, IEEE
 * add/sub/mul/div with no contraction (build with -ffp-contract=off), as
 * tack's LLVM codegen emits them (packages/tack-core/src/tack/codegen/
 * llvm_gen.py:589-591,621-639).  Rows are split across pthreads the way the
 * reference CPU backend fans a kernel's outer loop over a thread pool
 * (packages/tack-core/src/tack/runtime/cpu.py:530-744); the order of work
 * inside a row, and so every output byte, does not depend on the split.
 * Row offsets are int64 (the reference narrows numpy's int64 cumsum into
 * int32 fields; the values agree whenever they fit).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

typedef struct {
  int64_t nx, ny, nz;
  float x0, y0, z0, dx, dy, dz;
} orc_grid;

/* ---- a minimal parallel-for over [0, n) -------------------------------- */

typedef void (*range_fn)(void* ctx, int64_t lo, int64_t hi);

typedef struct {
  range_fn fn;
  void* ctx;
  int64_t lo, hi;
} range_job;

static void* range_worker(void* p) {
  range_job* j = (range_job*)p;
  j->fn(j->ctx, j->lo, j->hi);
  return NULL;
}

static int resolve_threads(int nthreads) {
  if (nthreads > 0) return nthreads;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

static void parallel_for(int64_t n, int nthreads, range_fn fn, void* ctx) {
  int t = resolve_threads(nthreads);
  if (t > 256) t = 256;
  if ((int64_t)t > n) t = (int)(n > 0 ? n : 1);
  if (t <= 1) {
    fn(ctx, 0, n);
    return;
  }
  pthread_t th[256];
  range_job jobs[256];
  for (int i = 0; i < t; ++i) {
    jobs[i].fn = fn;
    jobs[i].ctx = ctx;
    jobs[i].lo = n * i / t;
    jobs[i].hi = n * (i + 1) / t;
  }
  int started[256];
  for (int i = 1; i < t; ++i) started[i] = pthread_create(&th[i], NULL, range_worker, &jobs[i]) == 0;
  range_worker(&jobs[0]);
  for (int i = 1; i < t; ++i) {
    if (started[i])
      pthread_join(th[i], NULL);
    else
      range_worker(&jobs[i]);
  }
}

/* ---- grid helpers (UniformGrid.get_x/y/z, flying_edges.py:328-341) ----- */

static inline float gx(const orc_grid* g, int64_t i) { return g->x0 + (float)i * g->dx; }
static inline float gy(const orc_grid* g, int64_t j) { return g->y0 + (float)j * g->dy; }
static inline float gz(const orc_grid* g, int64_t k) { return g->z0 + (float)k * g->dz; }

/* ---- _fe_count_edges_xyz (flying_edges.py:399-437) ---------------------- */

typedef struct {
  const float* s;
  const orc_grid* g;
  float iso;
  int32_t *xc, *yc, *zc;
} count_edges_ctx;

static void count_edges_rows(void* p, int64_t lo, int64_t hi) {
  const count_edges_ctx* c = (const count_edges_ctx*)p;
  const orc_grid* g = c->g;
  const int64_t nx_p1 = g->nx + 1, ny_p1 = g->ny + 1, nxy_p1 = nx_p1 * ny_p1;
  const float iso = c->iso;
  for (int64_t row = lo; row < hi; ++row) {
    const int64_t j = row % ny_p1, k = row / ny_p1;
    const int64_t base = k * nxy_p1 + j * nx_p1;
    int32_t xc = 0, yc = 0, zc = 0;
    for (int64_t i = 0; i < nx_p1; ++i) {
      const float s = c->s[base + i];
      const int above = s > iso;
      if (i < g->nx) {
        const int a_nx = c->s[base + i + 1] > iso;
        if (above != a_nx) xc++;
      }
      if (j < g->ny) {
        const int a_ny = c->s[base + nx_p1 + i] > iso;
        if (above != a_ny) yc++;
      }
      if (k < g->nz) {
        const int a_nz = c->s[base + nxy_p1 + i] > iso;
        if (above != a_nz) zc++;
      }
    }
    c->xc[row] = xc;
    c->yc[row] = yc;
    c->zc[row] = zc;
  }
}

void orc_fe_count_edges_xyz(const float* s, const orc_grid* g, float iso, int32_t* row_xc,
                            int32_t* row_yc, int32_t* row_zc, int nthreads) {
  count_edges_ctx c = {s, g, iso, row_xc, row_yc, row_zc};
  parallel_for((g->ny + 1) * (g->nz + 1), nthreads, count_edges_rows, &c);
}

/* ---- _fe_count_rows (flying_edges.py:440-477) --------------------------- */

typedef struct {
  const float* s;
  const orc_grid* g;
  const int32_t* num_tris;
  const int32_t* mask;
  float iso;
  int32_t* tri;
} count_rows_ctx;

static void count_rows_rows(void* p, int64_t lo, int64_t hi) {
  const count_rows_ctx* c = (const count_rows_ctx*)p;
  const orc_grid* g = c->g;
  const int64_t nx_p1 = g->nx + 1, nxy_p1 = nx_p1 * (g->ny + 1);
  const float iso = c->iso;
  for (int64_t row = lo; row < hi; ++row) {
    const int64_t cj = row % g->ny, ck = row / g->ny;
    const int64_t base00 = ck * nxy_p1 + cj * nx_p1;
    const int64_t base10 = base00 + nx_p1, base01 = base00 + nxy_p1, base11 = base10 + nxy_p1;
    int32_t count = 0;
    float s0 = c->s[base00], s3 = c->s[base10], s4 = c->s[base01], s7 = c->s[base11];
    for (int64_t ci = 0; ci < g->nx; ++ci) {
      const float s1 = c->s[base00 + ci + 1], s2 = c->s[base10 + ci + 1];
      const float s5 = c->s[base01 + ci + 1], s6 = c->s[base11 + ci + 1];
      const int64_t cell_idx = ck * g->ny * g->nx + cj * g->nx + ci;
      if (!c->mask || c->mask[cell_idx] == 0) {
        int case_idx = 0;
        if (s0 > iso) case_idx += 1;
        if (s1 > iso) case_idx += 2;
        if (s2 > iso) case_idx += 4;
        if (s3 > iso) case_idx += 8;
        if (s4 > iso) case_idx += 16;
        if (s5 > iso) case_idx += 32;
        if (s6 > iso) case_idx += 64;
        if (s7 > iso) case_idx += 128;
        count += c->num_tris[case_idx];
      }
      s0 = s1;
      s3 = s2;
      s4 = s5;
      s7 = s6;
    }
    c->tri[row] = count;
  }
}

void orc_fe_count_rows(const float* s, const orc_grid* g, const int32_t* num_tris,
                       const int32_t* mask, float iso, int32_t* row_tri, int nthreads) {
  count_rows_ctx c = {s, g, num_tris, mask, iso, row_tri};
  parallel_for(g->ny * g->nz, nthreads, count_rows_rows, &c);
}

/* ---- _fe_emit_points_xyz (flying_edges.py:480-542) ---------------------- */

typedef struct {
  const float* s;
  const orc_grid* g;
  const int64_t *xo, *yo, *zo;
  float* points;
  float iso;
} emit_points_ctx;

static void emit_points_rows(void* p, int64_t lo, int64_t hi) {
  const emit_points_ctx* c = (const emit_points_ctx*)p;
  const orc_grid* g = c->g;
  const int64_t nx_p1 = g->nx + 1, ny_p1 = g->ny + 1, nxy_p1 = nx_p1 * ny_p1;
  const float iso = c->iso;
  float* pts = c->points;
  for (int64_t row = lo; row < hi; ++row) {
    const int64_t j = row % ny_p1, k = row / ny_p1;
    const int64_t base = k * nxy_p1 + j * nx_p1;
    int64_t xi = c->xo[row], yi = c->yo[row], zi = c->zo[row];
    for (int64_t i = 0; i < nx_p1; ++i) {
      const int64_t node = base + i;
      const float s = c->s[node];
      const int above = s > iso;
      const float px = gx(g, i), py = gy(g, j), pz = gz(g, k);
      if (i < g->nx) {
        const float s_n = c->s[node + 1];
        if (above != (s_n > iso)) {
          const float t = (iso - s) / (s_n - s + 1.0e-10f);
          const float px1 = gx(g, i + 1), py1 = gy(g, j), pz1 = gz(g, k);
          pts[xi * 3] = px + t * (px1 - px);
          pts[xi * 3 + 1] = py + t * (py1 - py);
          pts[xi * 3 + 2] = pz + t * (pz1 - pz);
          xi++;
        }
      }
      if (j < g->ny) {
        const float s_n = c->s[node + nx_p1];
        if (above != (s_n > iso)) {
          const float t = (iso - s) / (s_n - s + 1.0e-10f);
          const float px1 = gx(g, i), py1 = gy(g, j + 1), pz1 = gz(g, k);
          pts[yi * 3] = px + t * (px1 - px);
          pts[yi * 3 + 1] = py + t * (py1 - py);
          pts[yi * 3 + 2] = pz + t * (pz1 - pz);
          yi++;
        }
      }
      if (k < g->nz) {
        const float s_n = c->s[node + nxy_p1];
        if (above != (s_n > iso)) {
          const float t = (iso - s) / (s_n - s + 1.0e-10f);
          const float px1 = gx(g, i), py1 = gy(g, j), pz1 = gz(g, k + 1);
          pts[zi * 3] = px + t * (px1 - px);
          pts[zi * 3 + 1] = py + t * (py1 - py);
          pts[zi * 3 + 2] = pz + t * (pz1 - pz);
          zi++;
        }
      }
    }
  }
}

void orc_fe_emit_points_xyz(const float* s, const int64_t* row_xo, const int64_t* row_yo,
                            const int64_t* row_zo, float* points, const orc_grid* g, float iso,
                            int nthreads) {
  emit_points_ctx c = {s, g, row_xo, row_yo, row_zo, points, iso};
  parallel_for((g->ny + 1) * (g->nz + 1), nthreads, emit_points_rows, &c);
}

/* ---- _fe_emit_tris (flying_edges.py:545-656) ---------------------------- */

typedef struct {
  const float* s;
  const int64_t* tri_off;
  const int64_t *xo, *yo, *zo;
  int32_t* conn;
  const int32_t* mask;
  const orc_grid* g;
  const int32_t* tri_table;
  float iso;
} emit_tris_ctx;

static void emit_tris_rows(void* p, int64_t lo, int64_t hi) {
  const emit_tris_ctx* c = (const emit_tris_ctx*)p;
  const orc_grid* g = c->g;
  const int64_t nx_p1 = g->nx + 1, ny_p1 = g->ny + 1, nxy_p1 = nx_p1 * ny_p1;
  const float iso = c->iso;
  for (int64_t row = lo; row < hi; ++row) {
    const int64_t cj = row % g->ny, ck = row / g->ny;
    const int64_t r00 = ck * ny_p1 + cj, r10 = r00 + 1, r01 = r00 + ny_p1, r11 = r01 + 1;
    const int64_t xo00 = c->xo[r00], yo00 = c->yo[r00], zo00 = c->zo[r00];
    const int64_t xo10 = c->xo[r10], zo10 = c->zo[r10];
    const int64_t xo01 = c->xo[r01], yo01 = c->yo[r01];
    const int64_t xo11 = c->xo[r11];
    int64_t rx00 = 0, ry00 = 0, rz00 = 0, rx10 = 0, rz10 = 0, rx01 = 0, ry01 = 0, rx11 = 0;
    const int64_t base00 = ck * nxy_p1 + cj * nx_p1;
    const int64_t base10 = base00 + nx_p1, base01 = base00 + nxy_p1, base11 = base10 + nxy_p1;
    int64_t tri_idx = c->tri_off[row];
    float s0 = c->s[base00], s3 = c->s[base10], s4 = c->s[base01], s7 = c->s[base11];
    for (int64_t ci = 0; ci < g->nx; ++ci) {
      const float s1 = c->s[base00 + ci + 1], s2 = c->s[base10 + ci + 1];
      const float s5 = c->s[base01 + ci + 1], s6 = c->s[base11 + ci + 1];
      const int a0 = s0 > iso, a1 = s1 > iso, a2 = s2 > iso, a3 = s3 > iso;
      const int a4 = s4 > iso, a5 = s5 > iso, a6 = s6 > iso, a7 = s7 > iso;
      const int case_idx = a0 + a1 * 2 + a2 * 4 + a3 * 8 + a4 * 16 + a5 * 32 + a6 * 64 + a7 * 128;
      const int ix00 = a0 != a1, iy00 = a0 != a3, iz00 = a0 != a4;
      const int ix10 = a3 != a2, iz10 = a3 != a7;
      const int ix01 = a4 != a5, iy01 = a4 != a7;
      const int ix11 = a7 != a6;
      int64_t pid[12];
      pid[0] = xo00 + rx00;
      pid[1] = yo00 + ry00 + iy00;
      pid[2] = xo10 + rx10;
      pid[3] = yo00 + ry00;
      pid[4] = xo01 + rx01;
      pid[5] = yo01 + ry01 + iy01;
      pid[6] = xo11 + rx11;
      pid[7] = yo01 + ry01;
      pid[8] = zo00 + rz00;
      pid[9] = zo00 + rz00 + iz00;
      pid[10] = zo10 + rz10;
      pid[11] = zo10 + rz10 + iz10;
      rx00 += ix00;
      ry00 += iy00;
      rz00 += iz00;
      rx10 += ix10;
      rz10 += iz10;
      rx01 += ix01;
      ry01 += iy01;
      rx11 += ix11;
      const int64_t cell_idx = ck * g->ny * g->nx + cj * g->nx + ci;
      if (!c->mask || c->mask[cell_idx] == 0) {
        for (int t = 0; t < 16; t += 3) {
          const int e0 = c->tri_table[case_idx * 16 + t];
          if (e0 >= 0) {
            const int e1 = c->tri_table[case_idx * 16 + t + 1];
            const int e2 = c->tri_table[case_idx * 16 + t + 2];
            c->conn[tri_idx * 3] = (int32_t)pid[e0];
            c->conn[tri_idx * 3 + 1] = (int32_t)pid[e1];
            c->conn[tri_idx * 3 + 2] = (int32_t)pid[e2];
            tri_idx++;
          }
        }
      }
      s0 = s1;
      s3 = s2;
      s4 = s5;
      s7 = s6;
    }
  }
}

void orc_fe_emit_tris(const float* s, const int64_t* row_tri_offset, const int64_t* row_xo,
                      const int64_t* row_yo, const int64_t* row_zo, int32_t* conn,
                      const int32_t* mask, const orc_grid* g, const int32_t* tri_table, float iso,
                      int nthreads) {
  emit_tris_ctx c = {s, row_tri_offset, row_xo, row_yo, row_zo, conn, mask, g, tri_table, iso};
  parallel_for(g->ny * g->nz, nthreads, emit_tris_rows, &c);
}

/* ---- classify_cells (examples/26_marching_cubes.py:435-450) ------------- */

typedef struct {
  const float* s;
  const orc_grid* g;
  const int32_t* num_tris;
  float iso;
  uint8_t* cases;
  int32_t* ntri;
} classify_ctx;

static void classify_range(void* p, int64_t lo, int64_t hi) {
  const classify_ctx* c = (const classify_ctx*)p;
  const orc_grid* g = c->g;
  const int64_t nx_p1 = g->nx + 1, nxy_p1 = nx_p1 * (g->ny + 1), nxy = g->nx * g->ny;
  for (int64_t cell = lo; cell < hi; ++cell) {
    const int64_t ci = cell % g->nx, cj = (cell / g->nx) % g->ny, ck = cell / nxy;
    const int64_t b = ck * nxy_p1 + cj * nx_p1 + ci;
    const int64_t p[8] = {b, b + 1, b + nx_p1 + 1, b + nx_p1,
                          b + nxy_p1, b + nxy_p1 + 1, b + nxy_p1 + nx_p1 + 1, b + nxy_p1 + nx_p1};
    int case_idx = 0;
    for (int q = 0; q < 8; ++q)
      if (c->s[p[q]] > c->iso) case_idx += 1 << q;
    if (c->cases) c->cases[cell] = (uint8_t)case_idx;
    if (c->ntri) c->ntri[cell] = c->num_tris[case_idx];
  }
}

void orc_mc_classify_cells(const float* s, const orc_grid* g, const int32_t* num_tris, float iso,
                           uint8_t* cases, int32_t* ntri, int nthreads) {
  classify_ctx c = {s, g, num_tris, iso, cases, ntri};
  parallel_for(g->nx * g->ny * g->nz, nthreads, classify_range, &c);
}

/* ---- emit_triangles of examples/26_marching_cubes.py:453-503 ----------- */
/* The unmerged triangle soup: per cell, in cell order, the tri-table's
 * vertices interpolated between the edge's two corners, corner positions
 * from the cell's bounds (x_lo = x0 + float(ci)*dx, x_hi = x_lo + dx, corner
 * x = x_lo + cx * (x_hi - x_lo)), SoA out. */
static const float kCornerX[8] = {0, 1, 1, 0, 0, 1, 1, 0};
static const float kCornerY[8] = {0, 0, 1, 1, 0, 0, 1, 1};
static const float kCornerZ[8] = {0, 0, 0, 0, 1, 1, 1, 1};

typedef struct {
  const float* s;
  const orc_grid* g;
  const int32_t* tri_table;
  const int32_t* edge_corners;
  float iso;
  const int64_t* offsets;
  float *ox, *oy, *oz;
} soup_ctx;

static void soup_range(void* p, int64_t lo, int64_t hi) {
  const soup_ctx* c = (const soup_ctx*)p;
  const orc_grid* g = c->g;
  const int64_t nx_p1 = g->nx + 1, nxy_p1 = nx_p1 * (g->ny + 1), nxy = g->nx * g->ny;
  for (int64_t cell = lo; cell < hi; ++cell) {
    const int64_t ci = cell % g->nx, cj = (cell / g->nx) % g->ny, ck = cell / nxy;
    const int64_t b = ck * nxy_p1 + cj * nx_p1 + ci;
    const int64_t pt[8] = {b, b + 1, b + nx_p1 + 1, b + nx_p1,
                           b + nxy_p1, b + nxy_p1 + 1, b + nxy_p1 + nx_p1 + 1, b + nxy_p1 + nx_p1};
    float v[8];
    int case_idx = 0;
    for (int q = 0; q < 8; ++q) {
      v[q] = c->s[pt[q]];
      if (v[q] > c->iso) case_idx += 1 << q;
    }
    const float x_lo = g->x0 + (float)ci * g->dx, x_hi = x_lo + g->dx;
    const float y_lo = g->y0 + (float)cj * g->dy, y_hi = y_lo + g->dy;
    const float z_lo = g->z0 + (float)ck * g->dz, z_hi = z_lo + g->dz;
    int64_t out = c->offsets[cell] * 3;
    for (int t = 0; t < 16; ++t) {
      const int e = c->tri_table[case_idx * 16 + t];
      if (e < 0) continue;
      const int ca = c->edge_corners[2 * e], cb = c->edge_corners[2 * e + 1];
      const float va = v[ca], vb = v[cb];
      const float interp = (c->iso - va) / (vb - va + 1e-10f);
      const float xa = x_lo + kCornerX[ca] * (x_hi - x_lo), xb = x_lo + kCornerX[cb] * (x_hi - x_lo);
      const float ya = y_lo + kCornerY[ca] * (y_hi - y_lo), yb = y_lo + kCornerY[cb] * (y_hi - y_lo);
      const float za = z_lo + kCornerZ[ca] * (z_hi - z_lo), zb = z_lo + kCornerZ[cb] * (z_hi - z_lo);
      c->ox[out] = xa + interp * (xb - xa);
      c->oy[out] = ya + interp * (yb - ya);
      c->oz[out] = za + interp * (zb - za);
      ++out;
    }
  }
}

void orc_mc_soup(const float* s, const orc_grid* g, const int32_t* tri_table,
                 const int32_t* edge_corners, float iso, const int64_t* offsets, float* ox,
                 float* oy, float* oz, int nthreads) {
  soup_ctx c = {s, g, tri_table, edge_corners, iso, offsets, ox, oy, oz};
  parallel_for(g->nx * g->ny * g->nz, nthreads, soup_range, &c);
}

/* ---- exclusive_scan / inclusive_scan (scan.py:81-123), serial ---------- */

int64_t orc_scan_i32(const int32_t* in, int32_t* out, int64_t n, int inclusive) {
  int64_t run = 0;
  for (int64_t i = 0; i < n; ++i) {
    const int32_t x = in[i];
    out[i] = (int32_t)(uint32_t)(uint64_t)(inclusive ? run + x : run);
    run += x;
  }
  return run;
}

/* ---- Field.min/max/sum (field.py:116-134; cuda_backend.py:44-106) ------ */

void orc_reduce_f32(const float* v, int64_t n, double out4[4]) {
  float mn = INFINITY, mx = -INFINITY;
  double sum = 0.0;
  int64_t nan = 0;
  for (int64_t i = 0; i < n; ++i) {
    const float x = v[i];
    if (x != x) {
      nan++;
    } else {
      mn = fminf(mn, x);
      mx = fmaxf(mx, x);
    }
    sum += (double)x;
  }
  out4[0] = mn;
  out4[1] = mx;
  out4[2] = sum;
  out4[3] = (double)nan;
}

/* ---- compute_normals (compute_normals.py:16-90) ------------------------ */
/* Serial restatement: triangles in order, each area-weighted face normal
 * added to its three vertices in f32 (the reference adds them with atomics,
 * so its order, and its last-bit rounding, varies), then every vertex with
 * length > 1e-10 scaled by 1/length in f32. */
void orc_compute_normals(const float* p, const int32_t* conn, int64_t n_pts, int64_t n_tris,
                         float* out) {
  for (int64_t i = 0; i < 3 * n_pts; ++i) out[i] = 0.0f;
  for (int64_t t = 0; t < n_tris; ++t) {
    const int64_t i0 = conn[3 * t], i1 = conn[3 * t + 1], i2 = conn[3 * t + 2];
    const float e1x = p[3 * i1] - p[3 * i0], e1y = p[3 * i1 + 1] - p[3 * i0 + 1],
                e1z = p[3 * i1 + 2] - p[3 * i0 + 2];
    const float e2x = p[3 * i2] - p[3 * i0], e2y = p[3 * i2 + 1] - p[3 * i0 + 1],
                e2z = p[3 * i2 + 2] - p[3 * i0 + 2];
    const float nx = e1y * e2z - e1z * e2y;
    const float ny = e1z * e2x - e1x * e2z;
    const float nz = e1x * e2y - e1y * e2x;
    const int64_t ids[3] = {i0, i1, i2};
    for (int v = 0; v < 3; ++v) {
      out[3 * ids[v]] += nx;
      out[3 * ids[v] + 1] += ny;
      out[3 * ids[v] + 2] += nz;
    }
  }
  for (int64_t i = 0; i < n_pts; ++i) {
    const float x = out[3 * i], y = out[3 * i + 1], z = out[3 * i + 2];
    const float len = sqrtf(x * x + y * y + z * z);
    if (len > 1.0e-10f) {
      const float inv = 1.0f / len;
      out[3 * i] = x * inv;
      out[3 * i + 1] = y * inv;
      out[3 * i + 2] = z * inv;
    }
  }
}

int orc_num_threads(int nthreads) { return resolve_threads(nthreads); }
