/*
 * CPU oracle of the Gaussian rasterizer (forward compositing and backward).
 *
 * TEST INFRASTRUCTURE ONLY: tests compare the CUDA rasterizer with it; the
 * product never loads it.
 *
 * The reference patches a third-party renderer (graphdeco-inria/
 * diff-gaussian-rasterization @ 9c5c2028, not vendored in the reference) whose
 * arithmetic is therefore restated here from the published algorithms it
 * implements: 3D Gaussian Splatting (Kerbl et al. 2023) and EWA splatting
 * (Zwicker et al. 2001), with the conventions visible at the reference's call
 * sites (adapter.py:21-117, check.py:743-1052, prepare_native.py:8-29):
 * column-major view/projection matrices, quaternion (w, x, y, z), 0.3 px^2
 * screen low-pass with the optional opacity compensation, 3-sigma radius,
 * 16x16 tiles, alpha in [1/255, 0.99], stop below transmittance 1e-4, inverse
 * depth output, colour = SH + 0.5 clamped at 0.
 *
 * Everything is double precision. The pixel order per tile is the sort order
 * of the renderer: tile, then depth, then Gaussian index.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define TILE 16

typedef struct {
  double x, y, z;
} v3;

static v3 affine(const double* m, v3 p) {
  v3 r = {m[0] * p.x + m[4] * p.y + m[8] * p.z + m[12],
          m[1] * p.x + m[5] * p.y + m[9] * p.z + m[13],
          m[2] * p.x + m[6] * p.y + m[10] * p.z + m[14]};
  return r;
}

static double affine_w(const double* m, v3 p) {
  return m[3] * p.x + m[7] * p.y + m[11] * p.z + m[15];
}

/* Standard rotation matrix of q = (w, x, y, z), row-major. */
static void rot(const double* q, double R[9]) {
  double w = q[0], x = q[1], y = q[2], z = q[3];
  R[0] = 1 - 2 * (y * y + z * z); R[1] = 2 * (x * y - w * z); R[2] = 2 * (x * z + w * y);
  R[3] = 2 * (x * y + w * z); R[4] = 1 - 2 * (x * x + z * z); R[5] = 2 * (y * z - w * x);
  R[6] = 2 * (x * z - w * y); R[7] = 2 * (y * z + w * x); R[8] = 1 - 2 * (x * x + y * y);
}

static const double SH_C0 = 0.28209479177387814, SH_C1 = 0.4886025119029199;
static const double SH_C2[5] = {1.0925484305920792, -1.0925484305920792, 0.31539156525252005,
                                -1.0925484305920792, 0.5462742152960396};
static const double SH_C3[7] = {-0.5900435899266435, 2.890611442640554, -0.4570457994644658,
                                0.3731763325901154, -0.4570457994644658, 1.445305721320277,
                                -0.5900435899266435};

/* Basis values b[16] and their gradients g[16][3] wrt the unit direction. */
static void sh_basis(double x, double y, double z, double b[16], double g[16][3]) {
  double xx = x * x, yy = y * y, zz = z * z;
  memset(g, 0, sizeof(double) * 48);
  b[0] = SH_C0;
  b[1] = -SH_C1 * y; g[1][1] = -SH_C1;
  b[2] = SH_C1 * z; g[2][2] = SH_C1;
  b[3] = -SH_C1 * x; g[3][0] = -SH_C1;
  b[4] = SH_C2[0] * x * y; g[4][0] = SH_C2[0] * y; g[4][1] = SH_C2[0] * x;
  b[5] = SH_C2[1] * y * z; g[5][1] = SH_C2[1] * z; g[5][2] = SH_C2[1] * y;
  b[6] = SH_C2[2] * (2 * zz - xx - yy);
  g[6][0] = -2 * SH_C2[2] * x; g[6][1] = -2 * SH_C2[2] * y; g[6][2] = 4 * SH_C2[2] * z;
  b[7] = SH_C2[3] * x * z; g[7][0] = SH_C2[3] * z; g[7][2] = SH_C2[3] * x;
  b[8] = SH_C2[4] * (xx - yy); g[8][0] = 2 * SH_C2[4] * x; g[8][1] = -2 * SH_C2[4] * y;
  b[9] = SH_C3[0] * y * (3 * xx - yy);
  g[9][0] = 6 * SH_C3[0] * x * y; g[9][1] = 3 * SH_C3[0] * (xx - yy);
  b[10] = SH_C3[1] * x * y * z;
  g[10][0] = SH_C3[1] * y * z; g[10][1] = SH_C3[1] * x * z; g[10][2] = SH_C3[1] * x * y;
  b[11] = SH_C3[2] * y * (4 * zz - xx - yy);
  g[11][0] = -2 * SH_C3[2] * x * y; g[11][1] = SH_C3[2] * (4 * zz - xx - 3 * yy);
  g[11][2] = 8 * SH_C3[2] * y * z;
  b[12] = SH_C3[3] * z * (2 * zz - 3 * xx - 3 * yy);
  g[12][0] = -6 * SH_C3[3] * x * z; g[12][1] = -6 * SH_C3[3] * y * z;
  g[12][2] = SH_C3[3] * (6 * zz - 3 * xx - 3 * yy);
  b[13] = SH_C3[4] * x * (4 * zz - xx - yy);
  g[13][0] = SH_C3[4] * (4 * zz - 3 * xx - yy); g[13][1] = -2 * SH_C3[4] * x * y;
  g[13][2] = 8 * SH_C3[4] * x * z;
  b[14] = SH_C3[5] * z * (xx - yy);
  g[14][0] = 2 * SH_C3[5] * x * z; g[14][1] = -2 * SH_C3[5] * y * z; g[14][2] = SH_C3[5] * (xx - yy);
  b[15] = SH_C3[6] * x * (xx - 3 * yy);
  g[15][0] = 3 * SH_C3[6] * (xx - yy); g[15][1] = -6 * SH_C3[6] * x * y;
}

typedef struct {
  int P, degree, H, W, antialias;
  const double *bg, *means, *opacities, *scales, *rots, *view, *proj, *sh, *campos;
  double mod, tanx, tany;
} scene_t;

typedef struct {
  int visible, radius;
  double px, py, depth, conic[3], opacity, aa, rgb[3], cov3[6], A[6];
  double a0, b, c0;  /* screen covariance before the low-pass */
  int clampx, clampy, clamped[3];
  double tx, ty, tz, dir[3], dist;
} proj_t;

static void project(const scene_t* s, int i, proj_t* o) {
  memset(o, 0, sizeof(*o));
  v3 p = {s->means[3 * i], s->means[3 * i + 1], s->means[3 * i + 2]};
  v3 t = affine(s->view, p);
  if (t.z <= 0.2) return;
  double sc[3] = {s->mod * s->scales[3 * i], s->mod * s->scales[3 * i + 1],
                  s->mod * s->scales[3 * i + 2]};
  double R[9];
  rot(s->rots + 4 * i, R);
  /* Sigma = R diag(s^2) R^T */
  for (int r = 0, k = 0; r < 3; ++r)
    for (int c = r; c < 3; ++c, ++k) {
      double acc = 0;
      for (int j = 0; j < 3; ++j) acc += R[3 * r + j] * sc[j] * sc[j] * R[3 * c + j];
      o->cov3[k] = acc;
    }
  double W = s->W, H = s->H;
  double fx = W / (2 * s->tanx), fy = H / (2 * s->tany);
  double limx = 1.3 * s->tanx, limy = 1.3 * s->tany;
  double rx = t.x / t.z, ry = t.y / t.z;
  o->clampx = rx < -limx || rx > limx;
  o->clampy = ry < -limy || ry > limy;
  o->tx = fmin(limx, fmax(-limx, rx)) * t.z;
  o->ty = fmin(limy, fmax(-limy, ry)) * t.z;
  o->tz = t.z;
  double J00 = fx / t.z, J02 = -fx * o->tx / (t.z * t.z);
  double J11 = fy / t.z, J12 = -fy * o->ty / (t.z * t.z);
  for (int c = 0; c < 3; ++c) {
    /* camera rotation row r, column c = view[4c + r] */
    o->A[c] = J00 * s->view[4 * c] + J02 * s->view[4 * c + 2];
    o->A[3 + c] = J11 * s->view[4 * c + 1] + J12 * s->view[4 * c + 2];
  }
  double S[9] = {o->cov3[0], o->cov3[1], o->cov3[2], o->cov3[1], o->cov3[3], o->cov3[4],
                 o->cov3[2], o->cov3[4], o->cov3[5]};
  double q[2][2] = {{0, 0}, {0, 0}};
  for (int r = 0; r < 2; ++r)
    for (int c = 0; c < 2; ++c)
      for (int k = 0; k < 3; ++k)
        for (int l = 0; l < 3; ++l) q[r][c] += o->A[3 * r + k] * S[3 * k + l] * o->A[3 * c + l];
  o->a0 = q[0][0]; o->b = q[0][1]; o->c0 = q[1][1];
  double a = o->a0 + 0.3, c = o->c0 + 0.3;
  double det0 = o->a0 * o->c0 - o->b * o->b, det = a * c - o->b * o->b;
  o->aa = s->antialias ? sqrt(fmax(0.000025, det0 / det)) : 1.0;
  if (det == 0) return;
  double mid = 0.5 * (a + c), disc = sqrt(fmax(0.1, mid * mid - det));
  o->radius = (int)ceil(3 * sqrt(fmax(mid + disc, mid - disc)));
  double hw = affine_w(s->proj, p);
  v3 h = affine(s->proj, p);
  double iw = 1 / (hw + 0.0000001);
  o->px = ((h.x * iw + 1) * W - 1) * 0.5;
  o->py = ((h.y * iw + 1) * H - 1) * 0.5;
  int gx = (s->W + TILE - 1) / TILE, gy = (s->H + TILE - 1) / TILE;
  int x0 = (int)fmin(gx, fmax(0, (int)((o->px - o->radius) / TILE)));
  int y0 = (int)fmin(gy, fmax(0, (int)((o->py - o->radius) / TILE)));
  int x1 = (int)fmin(gx, fmax(0, (int)((o->px + o->radius + TILE - 1) / TILE)));
  int y1 = (int)fmin(gy, fmax(0, (int)((o->py + o->radius + TILE - 1) / TILE)));
  if ((x1 - x0) * (y1 - y0) == 0) { o->radius = 0; return; }
  o->conic[0] = c / det; o->conic[1] = -o->b / det; o->conic[2] = a / det;
  o->opacity = s->opacities[i] * o->aa;
  double d[3] = {p.x - s->campos[0], p.y - s->campos[1], p.z - s->campos[2]};
  o->dist = sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
  for (int k = 0; k < 3; ++k) o->dir[k] = d[k] / o->dist;
  double bb[16], gg[16][3];
  sh_basis(o->dir[0], o->dir[1], o->dir[2], bb, gg);
  int nt = (s->degree + 1) * (s->degree + 1);
  for (int ch = 0; ch < 3; ++ch) {
    double v = 0;
    for (int j = 0; j < nt; ++j) v += bb[j] * s->sh[48 * i + 3 * j + ch];
    v += 0.5;
    o->clamped[ch] = v < 0;
    o->rgb[ch] = fmax(v, 0);
  }
  o->depth = t.z;
  o->visible = 1;
}

static int in_tile(const scene_t* s, const proj_t* g, int tx, int ty) {
  int gx = (s->W + TILE - 1) / TILE, gy = (s->H + TILE - 1) / TILE;
  int x0 = (int)fmin(gx, fmax(0, (int)((g->px - g->radius) / TILE)));
  int y0 = (int)fmin(gy, fmax(0, (int)((g->py - g->radius) / TILE)));
  int x1 = (int)fmin(gx, fmax(0, (int)((g->px + g->radius + TILE - 1) / TILE)));
  int y1 = (int)fmin(gy, fmax(0, (int)((g->py + g->radius + TILE - 1) / TILE)));
  return tx >= x0 && tx < x1 && ty >= y0 && ty < y1;
}

static const proj_t* g_sort_base;
static int by_depth(const void* a, const void* b) {
  int i = *(const int*)a, j = *(const int*)b;
  float di = (float)g_sort_base[i].depth, dj = (float)g_sort_base[j].depth;
  if (di != dj) return di < dj ? -1 : 1;
  return i < j ? -1 : (i > j);
}

/* Adjoints of one pixel's compositing, in double, from the quantities the
 * forward stored: m contributors (front to back) with their alphas a[k], the
 * transmittance in front of each, Tin[k], and per-Gaussian scalars
 * g[k] = dL/dC . colour_k + dL/dinvdepth * invdepth_k. With the final
 * transmittance Tf and bgdot = dL/dC . bg, the colour is
 * C = sum_k c_k a_k Tin_k + Tf bg, Tin_{k+1} = Tin_k (1 - a_k), so
 *   dL/da_k = g_k Tin_k - (S_k + Tf bgdot) / (1 - a_k),
 *   S_k = sum_{i>k} g_i a_i Tin_i   (an explicit suffix sum here).
 * `mag` (when given) receives |g_k Tin_k| + (sum_{i>k} |g_i a_i Tin_i| +
 * |Tf bgdot|) / (1 - a_k): the size of every term summed into dL/da_k (its
 * conditioning); `suffix` is scratch of m + m entries. */
static void pixel_alpha_adjoints(int m, const double* a, const double* Tin, const double* g,
                                 double Tf, double bgdot, double* dalpha, double* mag,
                                 double* suffix) {
  double run = 0, size = 0;
  double* sizes = suffix + m;
  for (int k = m - 1; k >= 0; --k) {
    suffix[k] = run;
    sizes[k] = size;
    run += g[k] * a[k] * Tin[k];
    size += fabs(g[k] * a[k] * Tin[k]);
  }
  for (int k = 0; k < m; ++k) {
    double behind = suffix[k] + Tf * bgdot;
    dalpha[k] = g[k] * Tin[k] - behind / (1 - a[k]);
    if (mag) mag[k] = fabs(g[k] * Tin[k]) + (sizes[k] + fabs(Tf * bgdot)) / (1 - a[k]);
  }
}

/* The per-pixel share of one contributor's screen adjoints given dL/dalpha:
 * with u = dL/dp = o G dL/dalpha (p the Gaussian's exponent, the 0.99 cap
 * not differentiated), dL/dQ = -1/2 u d d^T (full matrix entries a, b, c),
 * dL/dmean = -u Q d (pixels; times W/2, H/2 for NDC), dL/do = G dL/dalpha. */
static void pixel_screen_adjoints(double dx, double dy, const double conic[3], double o,
                                  double G, double dal, double W, double H, double out[6]) {
  double u = o * G * dal;
  out[0] = -u * (conic[0] * dx + conic[1] * dy) * 0.5 * W;
  out[1] = -u * (conic[1] * dx + conic[2] * dy) * 0.5 * H;
  out[2] = -0.5 * u * dx * dx;
  out[3] = -0.5 * u * dx * dy;
  out[4] = -0.5 * u * dy * dy;
  out[5] = G * dal;
}

/* Sizes of the terms of pixel_screen_adjoints: the same products with
 * |dL/dalpha| replaced by the size `dal_size` of what it sums and every
 * product taken by absolute value. */
static void pixel_term_sizes(double dx, double dy, const double conic[3], double o, double G,
                             double dal_size, double W, double H, double out[6]) {
  double u = o * G * dal_size;
  out[0] = u * (fabs(conic[0] * dx) + fabs(conic[1] * dy)) * 0.5 * W;
  out[1] = u * (fabs(conic[1] * dx) + fabs(conic[2] * dy)) * 0.5 * H;
  out[2] = 0.5 * u * dx * dx;
  out[3] = 0.5 * u * fabs(dx * dy);
  out[4] = 0.5 * u * dy * dy;
  out[5] = G * dal_size;
}

/* Forward + (when dpix != NULL) backward of the whole image.
 * Gradient outputs (may be NULL in forward-only use) are accumulated. */
static void render(const scene_t* s, double* color, double* invdepth, int* radii,
                   const double* dpix, const double* dinv, double* dmean2d, double* dconic,
                   double* dop_scaled, double* dcolor, double* dinvdepth, double* const* mags) {
  proj_t* g = calloc((size_t)s->P, sizeof(proj_t));
  for (int i = 0; i < s->P; ++i) {
    project(s, i, &g[i]);
    if (radii) radii[i] = g[i].visible ? g[i].radius : 0;
  }
  int gx = (s->W + TILE - 1) / TILE, gy = (s->H + TILE - 1) / TILE;
  size_t cap = (size_t)(s->P > 0 ? s->P : 1);
  int* list = malloc(sizeof(int) * cap);
  int* used = malloc(sizeof(int) * cap);
  double* alpha = malloc(sizeof(double) * cap);
  double* Tin = malloc(sizeof(double) * cap);
  double* gk = malloc(sizeof(double) * cap);
  double* dal = malloc(sizeof(double) * cap);
  double* suffix = malloc(2 * sizeof(double) * cap);
  double* magk = malloc(sizeof(double) * cap);
  for (int ty = 0; ty < gy; ++ty)
    for (int tx = 0; tx < gx; ++tx) {
      int n = 0;
      for (int i = 0; i < s->P; ++i)
        if (g[i].visible && g[i].radius > 0 && in_tile(s, &g[i], tx, ty)) list[n++] = i;
      g_sort_base = g;
      qsort(list, (size_t)n, sizeof(int), by_depth);
      for (int py = ty * TILE; py < (ty + 1) * TILE && py < s->H; ++py)
        for (int px = tx * TILE; px < (tx + 1) * TILE && px < s->W; ++px) {
          int pix = py * s->W + px, m = 0, hw = s->H * s->W;
          double T = 1, C[3] = {0, 0, 0}, D = 0;
          for (int k = 0; k < n; ++k) {
            const proj_t* q = &g[list[k]];
            double dx = q->px - px, dy = q->py - py;
            double power = -0.5 * (q->conic[0] * dx * dx + q->conic[2] * dy * dy) -
                           q->conic[1] * dx * dy;
            if (power > 0) continue;
            double al = fmin(0.99, q->opacity * exp(power));
            if (al < 1.0 / 255.0) continue;
            double tt = T * (1 - al);
            if (tt < 0.0001) break;
            for (int ch = 0; ch < 3; ++ch) C[ch] += q->rgb[ch] * al * T;
            D += (1.0 / q->depth) * al * T;
            used[m] = list[k];
            alpha[m] = al;
            Tin[m] = T;
            ++m;
            T = tt;
          }
          for (int ch = 0; ch < 3; ++ch) color[ch * hw + pix] = C[ch] + T * s->bg[ch];
          if (invdepth) invdepth[pix] = D;
          if (!dpix) continue;
          double dp[3] = {dpix[pix], dpix[hw + pix], dpix[2 * hw + pix]};
          double di = dinv ? dinv[pix] : 0;
          double bgdot = s->bg[0] * dp[0] + s->bg[1] * dp[1] + s->bg[2] * dp[2];
          for (int k = 0; k < m; ++k) {
            const proj_t* q = &g[used[k]];
            gk[k] = q->rgb[0] * dp[0] + q->rgb[1] * dp[1] + q->rgb[2] * dp[2] +
                    di / q->depth;
          }
          pixel_alpha_adjoints(m, alpha, Tin, gk, T, bgdot, dal, mags ? magk : NULL, suffix);
          for (int k = 0; k < m; ++k) {
            int id = used[k];
            const proj_t* q = &g[id];
            double w = alpha[k] * Tin[k];
            for (int ch = 0; ch < 3; ++ch) dcolor[3 * id + ch] += w * dp[ch];
            if (dinvdepth) dinvdepth[id] += w * di;
            double dx = q->px - px, dy = q->py - py;
            double G = exp(-0.5 * (q->conic[0] * dx * dx + q->conic[2] * dy * dy) -
                           q->conic[1] * dx * dy);
            double sa[6];
            pixel_screen_adjoints(dx, dy, q->conic, q->opacity, G, dal[k], s->W, s->H, sa);
            dmean2d[3 * id] += sa[0];
            dmean2d[3 * id + 1] += sa[1];
            dconic[4 * id] += sa[2];
            dconic[4 * id + 1] += sa[3];
            dconic[4 * id + 3] += sa[4];
            dop_scaled[id] += sa[5];
            if (mags) {
              double sm[6];
              pixel_term_sizes(dx, dy, q->conic, q->opacity, G, magk[k], s->W, s->H, sm);
              mags[0][3 * id] += sm[0];
              mags[0][3 * id + 1] += sm[1];
              mags[1][4 * id] += sm[2];
              mags[1][4 * id + 1] += sm[3];
              mags[1][4 * id + 3] += sm[4];
              mags[2][id] += sm[5];
              for (int ch = 0; ch < 3; ++ch) mags[3][3 * id + ch] += fabs(w * dp[ch]);
              mags[4][id] += fabs(w * di);
            }
          }
        }
    }
  free(list);
  free(used);
  free(alpha);
  free(Tin);
  free(gk);
  free(dal);
  free(suffix);
  free(magk);
  free(g);
}

static scene_t make_scene(int P, int degree, const double* bg, const double* means,
                          const double* opacities, const double* scales, double mod,
                          const double* rots, const double* view, const double* proj,
                          double tanx, double tany, int H, int W, const double* sh,
                          const double* campos, int antialias) {
  scene_t s = {P, degree, H, W, antialias, bg, means, opacities, scales, rots, view, proj, sh,
               campos, mod, tanx, tany};
  return s;
}

void oracle_raster_forward(int P, int degree, const double* bg, const double* means,
                           const double* opacities, const double* scales, double mod,
                           const double* rots, const double* view, const double* proj,
                           double tanx, double tany, int H, int W, const double* sh,
                           const double* campos, int antialias, double* color,
                           double* invdepth, int* radii) {
  scene_t s = make_scene(P, degree, bg, means, opacities, scales, mod, rots, view, proj, tanx,
                         tany, H, W, sh, campos, antialias);
  render(&s, color, invdepth, radii, NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL);
}

/* Full backward. Outputs (zero-initialised by the caller, P-major like the
 * renderer's): dmean2d [P][3], dconic [P][4], dopacity [P], dcolor [P][3],
 * dinvdepth [P], dmeans [P][3], dcov3d [P][6], dsh [P][48], dscales [P][3],
 * drots [P][4]. */
/* Geometry backward of Gaussian i (visible) as a function of its pixel-stage
 * adjoints x[10] = (dL/dmean2D x, y (NDC), dL/dconic a, b, c (full-matrix
 * entries), dL/d(blended opacity), dL/dcolour r, g, b, dL/d(inverse depth)).
 * Writes y[65] = (dL/dopacity, dL/dmeans [3], dL/dcov3D [6], dL/dsh [48],
 * dL/dscales [3], dL/drotations [4]); y is linear in x. */
static void geometry_one(const scene_t* s, int i, const double* x, double* y) {
  const double *means = s->means, *opacities = s->opacities, *scales = s->scales,
               *rots = s->rots, *view = s->view, *proj = s->proj, *sh = s->sh;
  const double mod = s->mod, tanx = s->tanx, tany = s->tany;
  const int W = s->W, H = s->H, degree = s->degree, antialias = s->antialias;
  memset(y, 0, sizeof(double) * 65);
  proj_t q;
  project(s, i, &q);
  if (!q.visible) return;
    v3 p = {means[3 * i], means[3 * i + 1], means[3 * i + 2]};
    double a0 = q.a0, b = q.b, c0 = q.c0, a = a0 + 0.3, c = c0 + 0.3;
    double det0 = a0 * c0 - b * b, det = a * c - b * b;
    double dl_da = 0, dl_db = 0, dl_dc = 0;
    double dop = x[5];
    y[0] = dop * q.aa;
    if (antialias) {
      double r = det0 / det;
      if (r > 0.000025) {
        double dl_dr = dop * opacities[i] * 0.5 / sqrt(r);
        dl_da += dl_dr * (c0 * det - det0 * c) / (det * det);
        dl_db += dl_dr * (-2 * b * det + 2 * b * det0) / (det * det);
        dl_dc += dl_dr * (a0 * det - det0 * a) / (det * det);
      }
    }
    /* conic = inverse([[a, b], [b, c]]); dconic[1] is half the off-diagonal adjoint */
    double gx = x[2], gy = 2 * x[3], gz = x[4];
    double d2 = det * det;
    dl_da += (-c * c * gx + b * c * gy + (det - a * c) * gz) / d2;
    dl_dc += ((det - a * c) * gx + a * b * gy - a * a * gz) / d2;
    dl_db += (2 * b * c * gx - (det + 2 * b * b) * gy + 2 * a * b * gz) / d2;
    /* screen covariance q = A S A^T: symmetric S, unique entries */
    double S[9] = {q.cov3[0], q.cov3[1], q.cov3[2], q.cov3[1], q.cov3[3], q.cov3[4],
                   q.cov3[2], q.cov3[4], q.cov3[5]};
    const double *A0 = q.A, *A1 = q.A + 3;
    int k = 0;
    for (int r = 0; r < 3; ++r)
      for (int cc = r; cc < 3; ++cc, ++k) {
        double f = r == cc ? 1 : 2;
        double sb = r == cc ? A0[r] * A1[r] : A0[r] * A1[cc] + A0[cc] * A1[r];
        y[4 + k] += f * (A0[r] * A0[cc] * dl_da + A1[r] * A1[cc] * dl_dc) + sb * dl_db;
      }
    /* through A = J W to the camera-space mean */
    double dA0[3], dA1[3];
    for (int kk = 0; kk < 3; ++kk) {
      double s0 = 0, s1 = 0;
      for (int l = 0; l < 3; ++l) { s0 += S[3 * kk + l] * A0[l]; s1 += S[3 * kk + l] * A1[l]; }
      dA0[kk] = 2 * dl_da * s0 + dl_db * s1;
      dA1[kk] = dl_db * s0 + 2 * dl_dc * s1;
    }
    double dJ00 = 0, dJ02 = 0, dJ11 = 0, dJ12 = 0;
    for (int col = 0; col < 3; ++col) {
      dJ00 += dA0[col] * view[4 * col]; dJ02 += dA0[col] * view[4 * col + 2];
      dJ11 += dA1[col] * view[4 * col + 1]; dJ12 += dA1[col] * view[4 * col + 2];
    }
    double fx = W / (2 * tanx), fy = H / (2 * tany), z = q.tz;
    double dtx = (q.clampx ? 0 : 1) * -fx / (z * z) * dJ02;
    double dty = (q.clampy ? 0 : 1) * -fy / (z * z) * dJ12;
    double dtz = -fx / (z * z) * dJ00 - fy / (z * z) * dJ11 + 2 * fx * q.tx / (z * z * z) * dJ02 +
                 2 * fy * q.ty / (z * z * z) * dJ12;
    dtz += -x[9] / (z * z);
    double dm[3];
    for (int kk = 0; kk < 3; ++kk)
      dm[kk] = view[4 * kk] * dtx + view[4 * kk + 1] * dty + view[4 * kk + 2] * dtz;
    /* projective divide: ndc = h.xy / (h.w + 1e-7) */
    {
      double hw = affine_w(proj, p) + 0.0000001;
      v3 h = affine(proj, p);
      for (int kk = 0; kk < 3; ++kk) {
        dm[kk] += (proj[4 * kk] / hw - proj[4 * kk + 3] * h.x / (hw * hw)) * x[0] +
                  (proj[4 * kk + 1] / hw - proj[4 * kk + 3] * h.y / (hw * hw)) * x[1];
      }
    }
    /* SH colour */
    {
      double bb[16], gg[16][3];
      sh_basis(q.dir[0], q.dir[1], q.dir[2], bb, gg);
      int nt = (degree + 1) * (degree + 1);
      double gc[3], dd[3] = {0, 0, 0};
      for (int ch = 0; ch < 3; ++ch) gc[ch] = q.clamped[ch] ? 0 : x[6 + ch];
      for (int j = 0; j < nt; ++j) {
        double dot = 0;
        for (int ch = 0; ch < 3; ++ch) {
          y[10 + 3 * j + ch] += bb[j] * gc[ch];
          dot += sh[48 * i + 3 * j + ch] * gc[ch];
        }
        for (int kk = 0; kk < 3; ++kk) dd[kk] += gg[j][kk] * dot;
      }
      double ds = q.dir[0] * dd[0] + q.dir[1] * dd[1] + q.dir[2] * dd[2];
      for (int kk = 0; kk < 3; ++kk) dm[kk] += (dd[kk] - q.dir[kk] * ds) / q.dist;
    }
    for (int kk = 0; kk < 3; ++kk) y[1 + kk] += dm[kk];
    /* Sigma = R diag(s^2) R^T -> scale and rotation */
    {
      double G[9] = {y[4], 0.5 * y[5], 0.5 * y[6],
                     0.5 * y[5], y[7], 0.5 * y[8],
                     0.5 * y[6], 0.5 * y[8], y[9]};
      double sc[3] = {mod * scales[3 * i], mod * scales[3 * i + 1], mod * scales[3 * i + 2]};
      double R[9], M[9], dM[9], dR[9];
      rot(rots + 4 * i, R);
      for (int r = 0; r < 3; ++r)
        for (int cc = 0; cc < 3; ++cc) M[3 * r + cc] = R[3 * r + cc] * sc[cc];
      for (int r = 0; r < 3; ++r)
        for (int cc = 0; cc < 3; ++cc) {
          double acc = 0;
          for (int l = 0; l < 3; ++l) acc += G[3 * r + l] * M[3 * l + cc];
          dM[3 * r + cc] = 2 * acc;
        }
      for (int cc = 0; cc < 3; ++cc)
        y[58 + cc] += mod * (dM[cc] * R[cc] + dM[3 + cc] * R[3 + cc] + dM[6 + cc] * R[6 + cc]);
      for (int r = 0; r < 3; ++r)
        for (int cc = 0; cc < 3; ++cc) dR[3 * r + cc] = dM[3 * r + cc] * sc[cc];
      /* dR/dq: numerically exact central difference of the polynomial map
       * (degree 2, so the central difference is exact up to rounding). */
      double qv[4] = {rots[4 * i], rots[4 * i + 1], rots[4 * i + 2], rots[4 * i + 3]};
      for (int kq = 0; kq < 4; ++kq) {
        double qp[4], qm[4], Rp[9], Rm[9], h = 1e-3, acc = 0;
        memcpy(qp, qv, sizeof qp);
        memcpy(qm, qv, sizeof qm);
        qp[kq] += h;
        qm[kq] -= h;
        rot(qp, Rp);
        rot(qm, Rm);
        for (int l = 0; l < 9; ++l) acc += dR[l] * (Rp[l] - Rm[l]) / (2 * h);
        y[61 + kq] += acc;
      }
    }
  }

void oracle_raster_backward(int P, int degree, const double* bg, const double* means,
                            const double* opacities, const double* scales, double mod,
                            const double* rots, const double* view, const double* proj,
                            double tanx, double tany, int H, int W, const double* sh,
                            const double* campos, int antialias, const double* dpix,
                            const double* dinv, double* dmean2d, double* dconic,
                            double* dopacity, double* dcolor, double* dinvdepth,
                            double* dmeans, double* dcov3d, double* dsh, double* dscales,
                            double* drots) {
  scene_t s = make_scene(P, degree, bg, means, opacities, scales, mod, rots, view, proj, tanx,
                         tany, H, W, sh, campos, antialias);
  double* color = malloc(sizeof(double) * 3 * (size_t)H * W);
  double* dop_scaled = calloc((size_t)(P > 0 ? P : 1), sizeof(double));
  render(&s, color, NULL, NULL, dpix, dinv, dmean2d, dconic, dop_scaled, dcolor, dinvdepth,
         NULL);
  free(color);
  for (int i = 0; i < P; ++i) {
    double x[10] = {dmean2d[3 * i], dmean2d[3 * i + 1], dconic[4 * i], dconic[4 * i + 1],
                    dconic[4 * i + 3], dop_scaled[i], dcolor[3 * i], dcolor[3 * i + 1],
                    dcolor[3 * i + 2], dinvdepth[i]};
    double y[65];
    proj_t q;
    project(&s, i, &q);
    if (!q.visible) continue;
    geometry_one(&s, i, x, y);
    dopacity[i] = y[0];
    for (int k = 0; k < 3; ++k) dmeans[3 * i + k] += y[1 + k];
    for (int k = 0; k < 6; ++k) dcov3d[6 * i + k] += y[4 + k];
    for (int k = 0; k < 48; ++k) dsh[48 * i + k] += y[10 + k];
    for (int k = 0; k < 3; ++k) dscales[3 * i + k] += y[58 + k];
    for (int k = 0; k < 4; ++k) drots[4 * i + k] += y[61 + k];
  }
  free(dop_scaled);
}

/* The pixel stage of the backward with the sizes of its sums, and the
 * geometry stage as a per-Gaussian linear map, for tolerances that follow the
 * conditioning of each adjoint. Outputs (zeroed by the caller): the pixel
 * stage's adjoints x_mean2d [P][3] (NDC), x_conic [P][4], x_opacity [P] (of
 * the blended opacity), x_color [P][3], x_invdepth [P]; the same shapes
 * `size_*` holding the sums of absolute values of the terms added into each;
 * and jac [P][65][10], the geometry map of geometry_one (zero rows for
 * invisible Gaussians). */
void oracle_raster_backward_sized(int P, int degree, const double* bg, const double* means,
                                  const double* opacities, const double* scales, double mod,
                                  const double* rots, const double* view, const double* proj,
                                  double tanx, double tany, int H, int W, const double* sh,
                                  const double* campos, int antialias, const double* dpix,
                                  const double* dinv, double* x_mean2d, double* x_conic,
                                  double* x_opacity, double* x_color, double* x_invdepth,
                                  double* size_mean2d, double* size_conic, double* size_opacity,
                                  double* size_color, double* size_invdepth, double* jac) {
  scene_t s = make_scene(P, degree, bg, means, opacities, scales, mod, rots, view, proj, tanx,
                         tany, H, W, sh, campos, antialias);
  double* color = malloc(sizeof(double) * 3 * (size_t)H * W);
  double* const mags[5] = {size_mean2d, size_conic, size_opacity, size_color, size_invdepth};
  render(&s, color, NULL, NULL, dpix, dinv, x_mean2d, x_conic, x_opacity, x_color, x_invdepth,
         mags);
  free(color);
  for (int i = 0; i < P; ++i)
    for (int k = 0; k < 10; ++k) {
      double e[10] = {0}, y[65];
      e[k] = 1;
      geometry_one(&s, i, e, y);
      for (int r = 0; r < 65; ++r) jac[((size_t)i * 65 + r) * 10 + k] = y[r];
    }
}

/* Sensitivity of the geometry map to rounding-level perturbations: for each
 * of `draws` draws, every input of the map (means, scales, rotations,
 * opacities, SH coefficients, camera matrices and position, and the
 * pixel-stage adjoints x [P][10]) is multiplied by (1 + rel u), u uniform in
 * [-1, 1] from a fixed-seed generator, and spread [P][65] receives the
 * largest |y_perturbed - y| over the draws. A float evaluation of the map
 * behaves like an exact evaluation at inputs perturbed by a few ulps, so this
 * spread (with rel a few float ulps) sizes its rounding error, including
 * where exact cancellation makes an output zero. */
static double lcg_uniform(uint64_t* state) {
  *state = *state * 6364136223846793005ull + 1442695040888963407ull;
  return ((*state >> 11) * (1.0 / 9007199254740992.0)) * 2.0 - 1.0;
}

static double* perturbed(const double* v, size_t n, double rel, uint64_t* state) {
  double* out = malloc(sizeof(double) * (n ? n : 1));
  for (size_t k = 0; k < n; ++k) out[k] = v[k] * (1.0 + rel * lcg_uniform(state));
  return out;
}

void oracle_raster_geometry_spread(int P, int degree, const double* bg, const double* means,
                                   const double* opacities, const double* scales, double mod,
                                   const double* rots, const double* view, const double* proj,
                                   double tanx, double tany, int H, int W, const double* sh,
                                   const double* campos, int antialias, const double* x,
                                   double rel, int draws, double* spread) {
  scene_t s = make_scene(P, degree, bg, means, opacities, scales, mod, rots, view, proj, tanx,
                         tany, H, W, sh, campos, antialias);
  double* y0 = malloc(sizeof(double) * 65 * (size_t)(P ? P : 1));
  for (int i = 0; i < P; ++i) geometry_one(&s, i, x + 10 * (size_t)i, y0 + 65 * (size_t)i);
  memset(spread, 0, sizeof(double) * 65 * (size_t)P);
  uint64_t state = 0x9e3779b97f4a7c15ull;
  for (int d = 0; d < draws; ++d) {
    double* pm = perturbed(means, 3 * (size_t)P, rel, &state);
    double* po = perturbed(opacities, (size_t)P, rel, &state);
    double* ps = perturbed(scales, 3 * (size_t)P, rel, &state);
    double* pr = perturbed(rots, 4 * (size_t)P, rel, &state);
    double* pv = perturbed(view, 16, rel, &state);
    double* pp = perturbed(proj, 16, rel, &state);
    double* psh = perturbed(sh, 48 * (size_t)P, rel, &state);
    double* pc = perturbed(campos, 3, rel, &state);
    double* px = perturbed(x, 10 * (size_t)P, rel, &state);
    scene_t q = make_scene(P, degree, bg, pm, po, ps, mod, pr, pv, pp, tanx, tany, H, W, psh,
                           pc, antialias);
    for (int i = 0; i < P; ++i) {
      double y[65];
      geometry_one(&q, i, px + 10 * (size_t)i, y);
      for (int r = 0; r < 65; ++r) {
        double dev = fabs(y[r] - y0[65 * (size_t)i + r]);
        if (dev > spread[65 * (size_t)i + r]) spread[65 * (size_t)i + r] = dev;
      }
    }
    free(pm); free(po); free(ps); free(pr); free(pv); free(pp); free(psh); free(pc); free(px);
  }
  free(y0);
}

/* The scalar loss sum(dpix * colour) + sum(dinv * inverse depth), for
 * finite-difference checks of the backward. */
double oracle_raster_loss(int P, int degree, const double* bg, const double* means,
                          const double* opacities, const double* scales, double mod,
                          const double* rots, const double* view, const double* proj,
                          double tanx, double tany, int H, int W, const double* sh,
                          const double* campos, int antialias, const double* dpix,
                          const double* dinv) {
  double* color = malloc(sizeof(double) * 3 * (size_t)H * W);
  double* inv = malloc(sizeof(double) * (size_t)H * W);
  oracle_raster_forward(P, degree, bg, means, opacities, scales, mod, rots, view, proj, tanx,
                        tany, H, W, sh, campos, antialias, color, inv, NULL);
  double L = 0;
  for (int k = 0; k < 3 * H * W; ++k) L += dpix[k] * color[k];
  if (dinv)
    for (int k = 0; k < H * W; ++k) L += dinv[k] * inv[k];
  free(color);
  free(inv);
  return L;
}

/* ------------------------------------------------------------------------
 * Pixel stage of already projected 2D Gaussians on selected tiles (the
 * 1920x1080 pixel-backward configuration, checked on a sample of tiles).
 *
 * Inputs are the float32 values the CUDA path reads: mean2d [P][2] pixels,
 * conic_opacity [P][4] (a, b, c, opacity), rgb [P][3], depth [P], radii [P].
 * Each tile's list is built here from the 3-sigma rectangles (every Gaussian
 * whose rectangle covers the tile), ordered by (float depth, index); the
 * CUDA path keeps only tiles its alpha footprint reaches, and the extra
 * entries here contribute nothing. For the pixels of the `ntiles` tiles
 * listed in `tiles` (tile index ty * grid_x + tx) it writes colour [3][H][W]
 * and final transmittance [H][W], and accumulates the adjoints of every
 * Gaussian from those pixels only: dmean2d [P][2] (NDC, as the renderer
 * reports), dconic [P][3] (a, b, c), dopacity [P] (of the opacity the blend
 * used), dcolor [P][3]. mag_* (same shapes) accumulate the absolute values
 * of the per-pixel terms with both parts of dL/dalpha taken by size: the
 * size of what the float sums add up (their conditioning).
 *
 * Contribution decisions are taken in double; the CUDA path takes them in
 * float with a fast exponential, so a decision within rounding of its
 * threshold may go the other way there:
 *  - an alpha within 1e-5 (relative) of 1/255 or an exponent within 1e-6 of
 *    0: that Gaussian is flagged in `ambiguous` [P] (rare);
 *  - a transmittance stop within 1e-4 (relative) of 1e-4: the candidate at
 *    the stop may or may not contribute, which changes its own term and,
 *    through the transmittance left behind, every earlier contributor's
 *    dL/dalpha by at most (|g| + |bg . dL/dC|) alpha T / (1 - alpha_j) (the
 *    candidate's g, alpha, T). allow_* (same shapes as mag_*) accumulate
 *    these possible changes, carried to each adjoint like the term sizes.
 * The exponent p = -1/2 d^T Q d is evaluated exactly as the CUDA path
 * rounds it (float, the same products and fused multiply-adds, so the same
 * bits): for an elongated Gaussian its terms cancel heavily and that float
 * value, not the exact one, is what the renderer composites; the derivatives
 * of p are then taken exactly. What remains between the two is the fast
 * exponential and the product with the opacity (relative error of alpha_k at
 * most kappa_k = eps (|p_k| + 8), eps = 2^-24) and the float rounding of
 * 1 - alpha_k and of the transmittance product. Through the transmittance a
 * change of alpha_k moves every term of the pixel by at most
 * e_k = (kappa_k + 2 eps) / (1 - alpha_k) relative. These roundings are
 * independent, so their sum grows like the square root of their count:
 * E = sqrt(sum_k e_k^2) is its standard deviation, and the pixel's terms add
 * 4 E times their sizes to allow_* (four standard deviations; the worst case
 * sum_k e_k would make the bound hundreds of times looser than the errors
 * seen), and the stop margin is the larger of 1e-4 and 4 E.
 * Returns 0, or -1 when memory runs out. */
static const float* g_tile_depth;
static int by_float_depth(const void* a, const void* b) {
  int i = *(const int*)a, j = *(const int*)b;
  float di = g_tile_depth[i], dj = g_tile_depth[j];
  if (di != dj) return di < dj ? -1 : 1;
  return i < j ? -1 : (i > j);
}

/* p = -1/2 d^T Q d rounded as the CUDA path rounds it: the quadratic in dy
 * c2 dy^2 + c1 dy + c0 with c2 = -c/2, c1 = -(b dx), c0 = -((a dx) dx)/2, by
 * Horner's rule with fused multiply-adds (every product of float operands
 * rounded to float; fmaf rounds once). d = mean - pixel in float. */
static float float_form(const float* co, float dx, float dy) {
  float ax = co[0] * dx;
  float c0 = -0.5f * (ax * dx), c1 = -(co[1] * dx), c2 = -0.5f * co[2];
  return fmaf(fmaf(c2, dy, c1), dy, c0);
}

static void add_sizes(double* mean2d, double* conic, double* opacity, int id,
                      const double sm[6]) {
  mean2d[2 * id] += sm[0];
  mean2d[2 * id + 1] += sm[1];
  for (int e = 0; e < 3; ++e) conic[3 * id + e] += sm[2 + e];
  opacity[id] += sm[5];
}

int oracle_pixel_tiles(int P, const float* mean2d, const float* conic_opacity, const float* rgb,
                       const float* depth, const int* radii, int W, int H, const double* bg,
                       int ntiles, const int* tiles, const double* dpix, double* color,
                       double* final_t, double* dmean2d, double* dconic, double* dopacity,
                       double* dcolor, double* mag_mean2d, double* mag_conic,
                       double* mag_opacity, double* mag_color, double* allow_mean2d,
                       double* allow_conic, double* allow_opacity, double* allow_color,
                       unsigned char* ambiguous) {
  int gx = (W + TILE - 1) / TILE, gy = (H + TILE - 1) / TILE, hw = W * H;
  size_t cap = (size_t)(P > 0 ? P : 1);
  int* list = malloc(sizeof(int) * cap);
  int* used = malloc(sizeof(int) * cap);
  double* alpha = malloc(sizeof(double) * cap);
  double* Tin = malloc(sizeof(double) * cap);
  double* gk = malloc(sizeof(double) * cap);
  double* dal = malloc(sizeof(double) * cap);
  double* mag = malloc(sizeof(double) * cap);
  double* suffix = malloc(2 * sizeof(double) * cap);
  if (!list || !used || !alpha || !Tin || !gk || !dal || !mag || !suffix) {
    free(list); free(used); free(alpha); free(Tin); free(gk); free(dal); free(mag);
    free(suffix);
    return -1;
  }
  g_tile_depth = depth;
  for (int t = 0; t < ntiles; ++t) {
    int tx = tiles[t] % gx, ty = tiles[t] / gx, n = 0;
    if (ty >= gy) continue;
    for (int i = 0; i < P; ++i) {
      int r = radii[i];
      if (r <= 0) continue;
      double mx = mean2d[2 * i], my = mean2d[2 * i + 1];
      int x0 = (int)fmin(gx, fmax(0, (int)((mx - r) / TILE)));
      int y0 = (int)fmin(gy, fmax(0, (int)((my - r) / TILE)));
      int x1 = (int)fmin(gx, fmax(0, (int)((mx + r + TILE - 1) / TILE)));
      int y1 = (int)fmin(gy, fmax(0, (int)((my + r + TILE - 1) / TILE)));
      if (tx >= x0 && tx < x1 && ty >= y0 && ty < y1) list[n++] = i;
    }
    qsort(list, (size_t)n, sizeof(int), by_float_depth);
    for (int py = ty * TILE; py < (ty + 1) * TILE && py < H; ++py)
      for (int px = tx * TILE; px < (tx + 1) * TILE && px < W; ++px) {
        int pix = py * W + px, m = 0;
        int cand = -1, cand_m = 0;  /* a stop decision within rounding */
        double cand_alpha = 0, cand_T = 0, T = 1, C[3] = {0, 0, 0}, E2 = 0;
        const double eps = 1.0 / 16777216.0;
        for (int k = 0; k < n; ++k) {
          int id = list[k];
          const float* co = conic_opacity + 4 * id;
          double power = float_form(co, mean2d[2 * id] - (float)px,
                                    mean2d[2 * id + 1] - (float)py);
          double kappa = eps * (fabs(power) + 8);
          if (power > 0) continue;
          double al = fmin(0.99, (double)co[3] * exp(power));
          if (fabs(al * 255.0 - 1.0) <= 1e-5 + kappa) ambiguous[id] = 1;
          if (al < 1.0 / 255.0) continue;
          double tt = T * (1 - al);
          double e_k = (kappa + 2 * eps) / (1 - al);
          double margin = fmax(1e-4, 4 * sqrt(E2 + e_k * e_k));
          if (cand < 0 && fabs(tt / 0.0001 - 1.0) <= margin) {
            cand = id;
            cand_m = m;
            cand_alpha = al;
            cand_T = T;
          }
          if (tt < 0.0001) break;
          for (int ch = 0; ch < 3; ++ch) C[ch] += rgb[3 * id + ch] * al * T;
          used[m] = id;
          alpha[m] = al;
          Tin[m] = T;
          ++m;
          T = tt;
          E2 += e_k * e_k;
        }
        for (int ch = 0; ch < 3; ++ch) color[ch * hw + pix] = C[ch] + T * bg[ch];
        final_t[pix] = T;
        double dp[3] = {dpix[pix], dpix[hw + pix], dpix[2 * hw + pix]};
        double bgdot = bg[0] * dp[0] + bg[1] * dp[1] + bg[2] * dp[2];
        for (int k = 0; k < m; ++k) {
          const float* c = rgb + 3 * used[k];
          gk[k] = c[0] * dp[0] + c[1] * dp[1] + c[2] * dp[2];
        }
        pixel_alpha_adjoints(m, alpha, Tin, gk, T, bgdot, dal, mag, suffix);
        for (int k = 0; k < m; ++k) {
          int id = used[k];
          const float* co = conic_opacity + 4 * id;
          double q[3] = {co[0], co[1], co[2]};
          double w = alpha[k] * Tin[k];
          for (int ch = 0; ch < 3; ++ch) {
            dcolor[3 * id + ch] += w * dp[ch];
            mag_color[3 * id + ch] += fabs(w * dp[ch]);
          }
          double dx = (double)mean2d[2 * id] - px, dy = (double)mean2d[2 * id + 1] - py;
          double G = exp(float_form(co, mean2d[2 * id] - (float)px,
                                    mean2d[2 * id + 1] - (float)py));
          double sa[6], sm[6];
          pixel_screen_adjoints(dx, dy, q, co[3], G, dal[k], W, H, sa);
          pixel_term_sizes(dx, dy, q, co[3], G, mag[k], W, H, sm);
          dmean2d[2 * id] += sa[0];
          dmean2d[2 * id + 1] += sa[1];
          for (int e = 0; e < 3; ++e) dconic[3 * id + e] += sa[2 + e];
          dopacity[id] += sa[5];
          add_sizes(mag_mean2d, mag_conic, mag_opacity, id, sm);
          /* the float blend's own rounding: 4 E of every term */
          double spread = 4 * sqrt(E2);
          for (int e = 0; e < 6; ++e) sm[e] *= spread;
          add_sizes(allow_mean2d, allow_conic, allow_opacity, id, sm);
          for (int ch = 0; ch < 3; ++ch) allow_color[3 * id + ch] += spread * fabs(w * dp[ch]);
        }
        if (cand >= 0) {
          /* The candidate's own term (whether or not it was kept here) ... */
          const float* cc = rgb + 3 * cand;
          const float* co = conic_opacity + 4 * cand;
          double q[3] = {co[0], co[1], co[2]};
          double g = cc[0] * dp[0] + cc[1] * dp[1] + cc[2] * dp[2];
          double change = (fabs(g) + fabs(bgdot)) * cand_alpha * cand_T;
          double dx = (double)mean2d[2 * cand] - px, dy = (double)mean2d[2 * cand + 1] - py;
          double G = exp(float_form(co, mean2d[2 * cand] - (float)px,
                                    mean2d[2 * cand + 1] - (float)py));
          double sm[6];
          pixel_term_sizes(dx, dy, q, co[3], G,
                           fabs(g) * cand_T + fabs(cand_T * bgdot) / (1 - cand_alpha), W, H, sm);
          add_sizes(allow_mean2d, allow_conic, allow_opacity, cand, sm);
          for (int ch = 0; ch < 3; ++ch)
            allow_color[3 * cand + ch] += fabs(cand_alpha * cand_T * dp[ch]);
          /* ... and the change it makes to every contributor in front of it. */
          for (int k = 0; k < cand_m && k < m; ++k) {
            int id = used[k];
            const float* cj = conic_opacity + 4 * id;
            double qj[3] = {cj[0], cj[1], cj[2]};
            double djx = (double)mean2d[2 * id] - px, djy = (double)mean2d[2 * id + 1] - py;
            double Gj = exp(float_form(cj, mean2d[2 * id] - (float)px,
                                       mean2d[2 * id + 1] - (float)py));
            pixel_term_sizes(djx, djy, qj, cj[3], Gj, change / (1 - alpha[k]), W, H, sm);
            add_sizes(allow_mean2d, allow_conic, allow_opacity, id, sm);
          }
        }
      }
  }
  free(list); free(used); free(alpha); free(Tin); free(gk); free(dal); free(mag); free(suffix);
  return 0;
}

