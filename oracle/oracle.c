/*
 * CPU oracle for the per-Gaussian backward-and-update path.
 *
 * TEST INFRASTRUCTURE ONLY. This file restates the reference's arithmetic on
 * the CPU so the CUDA kernels can be checked against it. Nothing in the
 * product links, loads or calls it; tests/, the smoke check and bench.py's CPU
 * baseline leg use it as the checker.
 *
 * Restated from a-elrawy/clad-3dgs:
 *   sh_basis ............ SHGradientConsumer.cu:20-76 (basis, products xy/yz/xz)
 *   sh_basis gradient ... controls/ManualSH.cu:85-112 (d term / d direction)
 *   term coefficients ... controls/ManualSH.cu:107-111 (d term / d c = b * seed)
 *   lane rules .......... SHGradientConsumer.cu:169-217 (visibility, clamped
 *                         channels, inactive degrees, invisible-still-updates,
 *                         width-16 shuffle-tree order of the direction adjoint)
 *   direction VJP ....... SHGradientConsumer.cu:78-84 (d/dp of (p-c)/|p-c| . s)
 *   torch fused Adam .... SHGradientConsumer.cu:132-143
 *   float Adam / SGD .... SHGradientConsumer.cu:92-124
 *   split addressing .... SHGradientConsumer.cu:145-167
 *   quaternion VJP ...... controls/ManualActivations.cu:20-36
 *   scale/opacity VJP ... controls/ManualActivations.cu:94-100
 *   activation Adam ..... normalization.cu:70-77
 *   reference loss / FD . SHGradientConsumer.cu:404-433, 498-520
 *   position Adam ....... torch fused Adam on xyz with dm as gradient
 *   shard update ........ the data-parallel exchange: rank-ordered gradient
 *                         sum, the activation VJPs and torch fused Adam above
 *
 * Every float/double operation is evaluated on its own, left to right as
 * written (compiled with -ffp-contract=off, no FMA), which is the evaluation
 * order the CUDA kernels use.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define C0 0.28209479177387814f
#define C1 0.4886025119029199f
#define C2_0 1.0925484305920792f
#define C2_1 -1.0925484305920792f
#define C2_2 0.31539156525252005f
#define C2_3 -1.0925484305920792f
#define C2_4 0.5462742152960396f
#define C3_0 -0.5900435899266435f
#define C3_1 2.890611442640554f
#define C3_2 -0.4570457994644658f
#define C3_3 0.3731763325901154f
#define C3_4 -0.4570457994644658f
#define C3_5 1.445305721320277f
#define C3_6 -0.5900435899266435f

typedef struct {
  float x, y, z, r, xx, yy, zz, xy, yz, xz;
} dir_t;

static dir_t direction(const float* p, const float* c) {
  dir_t d;
  float ux = p[0] - c[0], uy = p[1] - c[1], uz = p[2] - c[2];
  d.r = sqrtf((ux * ux + uy * uy) + uz * uz);
  d.x = ux / d.r;
  d.y = uy / d.r;
  d.z = uz / d.r;
  d.xx = d.x * d.x;
  d.yy = d.y * d.y;
  d.zz = d.z * d.z;
  d.xy = d.x * d.y;
  d.yz = d.y * d.z;
  d.xz = d.x * d.z;
  return d;
}

/* b_j(dir) and its gradient wrt the three direction components. */
static void basis(int j, const dir_t* d, float* b, float g[3]) {
  const float g9x = (float)(6.0 * (double)C3_0), g9y = (float)(3.0 * (double)C3_0);
  const float g12 = (float)(-6.0 * (double)C3_3);
  const float g15x = (float)(3.0 * (double)C3_6), g15y = (float)(-6.0 * (double)C3_6);
  g[0] = g[1] = g[2] = 0.f;
  switch (j) {
    case 0: *b = C0; break;
    case 1: *b = -C1 * d->y; g[1] = -C1; break;
    case 2: *b = C1 * d->z; g[2] = C1; break;
    case 3: *b = -C1 * d->x; g[0] = -C1; break;
    case 4: *b = C2_0 * d->xy; g[0] = C2_0 * d->y; g[1] = C2_0 * d->x; break;
    case 5: *b = C2_1 * d->yz; g[1] = C2_1 * d->z; g[2] = C2_1 * d->y; break;
    case 6:
      *b = C2_2 * ((2.f * d->zz - d->xx) - d->yy);
      g[0] = (-2.f * C2_2) * d->x;
      g[1] = (-2.f * C2_2) * d->y;
      g[2] = (4.f * C2_2) * d->z;
      break;
    case 7: *b = C2_3 * d->xz; g[0] = C2_3 * d->z; g[2] = C2_3 * d->x; break;
    case 8:
      *b = C2_4 * (d->xx - d->yy);
      g[0] = (2.f * C2_4) * d->x;
      g[1] = (-2.f * C2_4) * d->y;
      break;
    case 9:
      *b = (C3_0 * d->y) * (3.f * d->xx - d->yy);
      g[0] = g9x * d->xy;
      g[1] = g9y * (d->xx - d->yy);
      break;
    case 10:
      *b = (C3_1 * d->xy) * d->z;
      g[0] = C3_1 * d->yz;
      g[1] = C3_1 * d->xz;
      g[2] = C3_1 * d->xy;
      break;
    case 11:
      *b = (C3_2 * d->y) * ((4.f * d->zz - d->xx) - d->yy);
      g[0] = (-2.0f * C3_2) * d->xy;
      g[1] = C3_2 * ((4.f * d->zz - d->xx) - 3.f * d->yy);
      g[2] = (8.0f * C3_2) * d->yz;
      break;
    case 12:
      *b = (C3_3 * d->z) * ((2.f * d->zz - 3.f * d->xx) - 3.f * d->yy);
      g[0] = g12 * d->xz;
      g[1] = g12 * d->yz;
      g[2] = C3_3 * ((6.f * d->zz - 3.f * d->xx) - 3.f * d->yy);
      break;
    case 13:
      *b = (C3_4 * d->x) * ((4.f * d->zz - d->xx) - d->yy);
      g[0] = C3_4 * ((4.f * d->zz - 3.f * d->xx) - d->yy);
      g[1] = (-2.0f * C3_4) * d->xy;
      g[2] = (8.0f * C3_4) * d->xz;
      break;
    case 14:
      *b = (C3_5 * d->z) * (d->xx - d->yy);
      g[0] = (2.0f * C3_5) * d->xz;
      g[1] = (-(2.0f * C3_5)) * d->yz;
      g[2] = C3_5 * (d->xx - d->yy);
      break;
    default:
      *b = (C3_6 * d->x) * (d->xx - 3.f * d->yy);
      g[0] = g15x * (d->xx - d->yy);
      g[1] = g15y * d->xy;
      break;
  }
}

static void torch_adam(float* p, float* m, float* v, float g, float step,
                       float bias2) {
  const double gd = (double)g;
  *m = (float)(0.9 * (double)*m + (1.0 - 0.9) * gd);
  *v = (float)(0.999 * (double)*v + ((1.0 - 0.999) * gd) * gd);
  const float denom = (float)((double)(sqrtf(*v) / bias2) + 1e-15);
  *p = *p - (step * *m) / denom;
}

static void float_adam(float* p, float* m, float* v, float g, float rate,
                       float inv1, float inv2) {
  *m = 0.9f * *m + 0.1f * g;
  *v = 0.999f * *v + (0.001f * g) * g;
  *p = *p - (rate * (*m * inv1)) / (sqrtf(*v * inv2) + 1e-15f);
}

/* mode: 0 SGD (packed coeff), 1 Adam (packed coeff/first/second, AdamConfig),
 *       2 split Adam (AdamConfig), 3 split torch Adam (TorchAdamConfig).
 * coefficient: optional packed [n][48] snapshot for the split modes. */
void oracle_sh_consume(int mode, int64_t n, int degree, const float* means,
                       const int* radii, const uint8_t* clamped,
                       const float* camera, const float* seed, float* dm,
                       const float* coefficient, float* coeff, float* first,
                       float* second, float* dc, float* rest, float* dc_first,
                       float* dc_second, float* rest_first, float* rest_second,
                       float bias1, float bias2_sqrt, float inv_bias1,
                       float inv_bias2) {
  const int nterms = (degree + 1) * (degree + 1);
  const float step_dc = (float)(0.0025 / (double)bias1);
  const float step_rest = (float)(0.000125 / (double)bias1);
  for (int64_t i = 0; i < n; ++i) {
    const int visible = radii[i] > 0;
    if (mode == 0 && !visible) continue; /* SGD does not update invisible */
    float s[3] = {0.f, 0.f, 0.f};
    dir_t d;
    memset(&d, 0, sizeof d);
    if (visible) {
      d = direction(means + 3 * i, camera);
      for (int ch = 0; ch < 3; ++ch)
        s[ch] = clamped[3 * i + ch] ? 0.f : seed[3 * i + ch];
    }
    float t[16][3];
    for (int j = 0; j < 16; ++j) {
      float g[3] = {0.f, 0.f, 0.f};
      t[j][0] = t[j][1] = t[j][2] = 0.f;
      const int split = mode >= 2;
      float *pp, *mm = NULL, *vv = NULL;
      if (split) {
        pp = j == 0 ? dc + 3 * i : rest + 45 * i + 3 * (j - 1);
        mm = j == 0 ? dc_first + 3 * i : rest_first + 45 * i + 3 * (j - 1);
        vv = j == 0 ? dc_second + 3 * i : rest_second + 45 * i + 3 * (j - 1);
      } else {
        pp = coeff + 48 * i + 3 * j;
        if (mode == 1) {
          mm = first + 48 * i + 3 * j;
          vv = second + 48 * i + 3 * j;
        }
      }
      if (visible && j < nterms) {
        float b, gr[3];
        basis(j, &d, &b, gr);
        const float* c = (split && coefficient) ? coefficient + 48 * i + 3 * j : pp;
        const float dot = (c[0] * s[0] + c[1] * s[1]) + c[2] * s[2];
        for (int k = 0; k < 3; ++k) t[j][k] = gr[k] * dot;
        for (int ch = 0; ch < 3; ++ch) g[ch] = b * s[ch];
      }
      for (int ch = 0; ch < 3; ++ch) {
        switch (mode) {
          case 0: pp[ch] = pp[ch] - 1e-3f * g[ch]; break;
          case 1:
          case 2:
            float_adam(pp + ch, mm + ch, vv + ch, g[ch],
                       j == 0 ? 0.0025f : 0.000125f, inv_bias1, inv_bias2);
            break;
          default:
            torch_adam(pp + ch, mm + ch, vv + ch, g[ch],
                       j == 0 ? step_dc : step_rest, bias2_sqrt);
        }
      }
    }
    if (!visible) continue;
    float total[3];
    for (int k = 0; k < 3; ++k) {
      float v[4];
      for (int r = 0; r < 4; ++r)
        v[r] = (t[r][k] + t[r + 8][k]) + (t[r + 4][k] + t[r + 12][k]);
      total[k] = (v[0] + v[2]) + (v[1] + v[3]);
    }
    const float ds = (d.x * total[0] + d.y * total[1]) + d.z * total[2];
    dm[3 * i + 0] = dm[3 * i + 0] + (total[0] - d.x * ds) / d.r;
    dm[3 * i + 1] = dm[3 * i + 1] + (total[1] - d.y * ds) / d.r;
    dm[3 * i + 2] = dm[3 * i + 2] + (total[2] - d.z * ds) / d.r;
  }
}

static float quaternion_component(const float* q, const float* s, float norm,
                                  int k) {
  if (norm < 1e-12f) return s[k] / 1e-12f;
  float dot = 0.f;
  for (int j = 0; j < 4; ++j) dot = dot + (q[j] / norm) * s[j];
  return (s[k] - (q[k] / norm) * dot) / norm;
}

void oracle_quaternion_backward(int64_t n, const float* q, const float* seed,
                                const float* norms, float* out) {
  for (int64_t i = 0; i < n; ++i)
    for (int k = 0; k < 4; ++k)
      out[4 * i + k] = quaternion_component(q + 4 * i, seed + 4 * i, norms[i], k);
}

/* params/seeds/first/second: [0] rotation n x 4, [1] scaling n x 3,
 * [2] opacity n x 1; saved: norm n, exp(scaling) n x 3, sigmoid(opacity) n. */
void oracle_activation_consume(int64_t n, float* const* params,
                               const float* const* seeds,
                               const float* const* saved, float* const* first,
                               float* const* second, const double* rates,
                               const float* bias1, const float* bias2) {
  float step[3];
  for (int j = 0; j < 3; ++j) step[j] = (float)(rates[j] / (double)bias1[j]);
  for (int64_t i = 0; i < n; ++i) {
    float g[4];
    for (int k = 0; k < 4; ++k)
      g[k] = quaternion_component(params[0] + 4 * i, seeds[0] + 4 * i,
                                  saved[0][i], k);
    for (int k = 0; k < 4; ++k)
      torch_adam(params[0] + 4 * i + k, first[0] + 4 * i + k,
                 second[0] + 4 * i + k, g[k], step[0], bias2[0]);
    for (int k = 0; k < 3; ++k)
      torch_adam(params[1] + 3 * i + k, first[1] + 3 * i + k,
                 second[1] + 3 * i + k, saved[1][3 * i + k] * seeds[1][3 * i + k],
                 step[1], bias2[1]);
    const float a = saved[2][i];
    torch_adam(params[2] + i, first[2] + i, second[2] + i,
               (a * (1.f - a)) * seeds[2][i], step[2], bias2[2]);
  }
}

/* Torch-fused Adam on positions [n][3] with dm as the gradient (no reference
 * counterpart; the same update as torch_adam above, every element). */
void oracle_xyz_adam(int64_t n, float* means, const float* dm, float* first,
                     float* second, double rate, float bias1, float bias2) {
  const float step = (float)(rate / (double)bias1);
  for (int64_t e = 0; e < 3 * n; ++e)
    torch_adam(means + e, first + e, second + e, dm[e], step, bias2);
}

/* Data-parallel exchange + update of the Gaussians [begin, end) (no
 * reference counterpart; it combines the activation VJPs and torch-fused Adam
 * above with a rank-ordered sum of per-view gradients). Groups g = 0..4 are
 * xyz [.,3], sh [.,48], scaling [.,3], rotation [.,4], opacity [.,1];
 * grads[q * 5 + g] start at Gaussian grad_origin, params[g] and the saved
 * arrays at 0, first/second[g] at begin. rates: xyz, f_dc, f_rest, scaling,
 * rotation, opacity. */
void oracle_shard_update(int64_t begin, int64_t end, int64_t grad_origin,
                         int ranks, const float* const* grads,
                         float* const* params, float* const* first,
                         float* const* second, const float* saved_scaling,
                         const float* saved_opacity, const float* saved_norm,
                         const double* rates, float bias1, float bias2) {
  static const int width[5] = {3, 48, 3, 4, 1};
  float step[6];
  for (int r = 0; r < 6; ++r) step[r] = (float)(rates[r] / (double)bias1);
  for (int g = 0; g < 5; ++g) {
    const int k = width[g];
    for (int64_t i = begin; i < end; ++i) {
      float sum[48];
      for (int c = 0; c < k; ++c) {
        const int64_t e = (i - grad_origin) * k + c;
        float s = grads[g][e];
        for (int q = 1; q < ranks; ++q) s = s + grads[q * 5 + g][e];
        sum[c] = s;
      }
      float grad[48];
      float* p = params[g] + i * k;
      for (int c = 0; c < k; ++c) {
        if (g == 2)
          grad[c] = saved_scaling[3 * i + c] * sum[c];
        else if (g == 4)
          grad[c] = (saved_opacity[i] * (1.f - saved_opacity[i])) * sum[c];
        else if (g == 3)
          grad[c] = quaternion_component(p, sum, saved_norm[i], c);
        else
          grad[c] = sum[c];
      }
      for (int c = 0; c < k; ++c) {
        const float st = g == 1 ? (c < 3 ? step[1] : step[2])
                                : step[g == 0 ? 0 : g + 1];
        const int64_t m = (i - begin) * k + c;
        torch_adam(p + c, first[g] + m, second[g] + m, grad[c], st, bias2);
      }
    }
  }
}

/* The reference's double-precision loss: sum_j b_j(dir) (c_j . w), with the
 * basis constants rounded to float first as the reference does. */
static double reference_loss(const double* p, const double* c, const double* w,
                             const float* camera, int degree) {
  double dx = p[0] - camera[0], dy = p[1] - camera[1], dz = p[2] - camera[2];
  double r = sqrt(dx * dx + dy * dy + dz * dz);
  double x = dx / r, y = dy / r, z = dz / r;
  double xx = x * x, yy = y * y, zz = z * z;
  double b[16];
  b[0] = (double)C0;
  b[1] = -(double)C1 * y;
  b[2] = (double)C1 * z;
  b[3] = -(double)C1 * x;
  b[4] = (double)C2_0 * x * y;
  b[5] = (double)C2_1 * y * z;
  b[6] = (double)C2_2 * (2 * zz - xx - yy);
  b[7] = (double)C2_3 * x * z;
  b[8] = (double)C2_4 * (xx - yy);
  b[9] = (double)C3_0 * y * (3 * xx - yy);
  b[10] = (double)C3_1 * x * y * z;
  b[11] = (double)C3_2 * y * (4 * zz - xx - yy);
  b[12] = (double)C3_3 * z * (2 * zz - 3 * xx - 3 * yy);
  b[13] = (double)C3_4 * x * (4 * zz - xx - yy);
  b[14] = (double)C3_5 * z * (xx - yy);
  b[15] = (double)C3_6 * x * (xx - 3 * yy);
  double result = 0;
  for (int j = 0; j < (degree + 1) * (degree + 1); ++j)
    result += b[j] * (c[3 * j] * w[0] + c[3 * j + 1] * w[1] + c[3 * j + 2] * w[2]);
  return result;
}

/* Central finite differences (step h) of reference_loss wrt the 3 position
 * components and the 48 coefficients of every visible Gaussian; out is n x 51
 * (zeros for invisible Gaussians). weights are the clamped seeds. */
void oracle_sh_fd_gradient(int64_t n, int degree, const float* means,
                           const int* radii, const float* coeff,
                           const float* weights, const float* camera, double h,
                           double* out) {
  for (int64_t i = 0; i < n; ++i) {
    double* row = out + 51 * i;
    for (int k = 0; k < 51; ++k) row[k] = 0;
    if (radii[i] <= 0) continue;
    double p[3], c[48], w[3];
    for (int k = 0; k < 3; ++k) {
      p[k] = means[3 * i + k];
      w[k] = weights[3 * i + k];
    }
    for (int k = 0; k < 48; ++k) c[k] = coeff[48 * i + k];
    for (int k = 0; k < 51; ++k) {
      double* value = k < 3 ? p + k : c + k - 3;
      const double old = *value;
      *value = old + h;
      const double plus = reference_loss(p, c, w, camera, degree);
      *value = old - h;
      const double minus = reference_loss(p, c, w, camera, degree);
      *value = old;
      row[k] = (plus - minus) / (2 * h);
    }
  }
}
