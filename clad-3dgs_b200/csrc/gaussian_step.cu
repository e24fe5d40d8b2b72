// Per-Gaussian backward-and-update kernels for B200 (sm_100a).
//
// One kernel template covers the reference's SH consumer (all four update
// modes, SHGradientConsumer.cu:92-217), the activation consumer
// (normalization.cu:79-101) and the fused pass that does both. Data layout and
// schedule:
//
//  * Gaussians are processed in tiles of kTile = 32. For each tile every array
//    the mode touches (means, radii, clamped, seeds, dm, dc/rest and their two
//    moments, activation parameters/moments/seeds/saved values) is one
//    contiguous byte range in HBM, so a tile is fetched with one 1D bulk copy
//    (cp.async.bulk, the TMA engine) per array into shared memory and written
//    back the same way. There are no per-lane 12-byte accesses.
//  * The main kernel is persistent: up to three CTAs per SM, each with a ring of
//    stages in shared memory, one producer warp issuing the bulk loads ahead
//    and the bulk stores behind, and sixteen consumer warps doing the
//    arithmetic. The consumers signal each computed tile on an mbarrier and
//    never wait on a store; the producer stores that tile, waits until the
//    stores have read the stage and refills it. HBM reads, compute and HBM
//    writes overlap, and one CTA's barrier waits overlap another's arithmetic.
//  * Per tile: the view direction of each Gaussian is computed once (phase A0),
//    warp j then owns SH term j for the 32 Gaussians of the tile (phase A1, lane
//    = Gaussian, compile-time term, no divergent switch), and all consumers run
//    one compact Adam update per parameter element (phase B). See "Arithmetic on
//    one staged tile" below.
//  * The tail tile and inputs that are not 16-byte aligned go through a plain
//    one-tile-per-CTA kernel with the same arithmetic.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <utility>

#include "async_copy.cuh"
#include "gaussian_math.cuh"
#include "clad3dgs_b200.h"

namespace clad3dgs {

// Per-module fault word written by bounded waits that gave up.
__device__ unsigned int g_fault_word = 0;

// ---------------------------------------------------------------------------
// Arrays a tile can stage. Widths are per Gaussian; CLAMPED is one byte per
// element, everything else four.
enum Arr : int {
  MEANS, RADII, CLAMPED, SEED, DM,
  // Updated parameters, then first moments, then second moments: every tile
  // slice is a multiple of 128 bytes, so each group is one contiguous region of
  // the stage and phase B walks it with a single index.
  DC, REST, COEF, ROT, SCL, OPA,
  DC_M, REST_M, COEF_M, ROT_M, SCL_M, OPA_M,
  DC_V, REST_V, COEF_V, ROT_V, SCL_V, OPA_V,
  SNAP, SEED_ROT, SEED_SCL, SEED_OPA, SAVED_NORM, SAVED_SCL, SAVED_OPA,
  // Adam moments of the positions (means are then updated and written back).
  XYZ_M, XYZ_V,
  NUM_ARR
};

constexpr int kWidth[NUM_ARR] = {3, 1, 3, 3, 3,
                                 3, 45, 48, 4, 3, 1,
                                 3, 45, 48, 4, 3, 1,
                                 3, 45, 48, 4, 3, 1,
                                 48, 4, 3, 1, 1, 3, 1,
                                 3, 3};
constexpr bool kWritten[NUM_ARR] = {0, 0, 0, 0, 1,
                                    1, 1, 1, 1, 1, 1,
                                    1, 1, 1, 1, 1, 1,
                                    1, 1, 1, 1, 1, 1,
                                    0, 0, 0, 0, 0, 0, 0,
                                    1, 1};
constexpr int elem_bytes(int a) { return a == CLAMPED ? 1 : 4; }

enum ShMode : int { SH_NONE, SH_SGD, SH_ADAM, SH_SPLIT_ADAM, SH_SPLIT_TORCH };

// Tile size and resident persistent CTAs per SM. Several independent CTAs per
// SM let one CTA's barrier waits overlap another's arithmetic.
#ifndef CLAD3DGS_TILE
#define CLAD3DGS_TILE 32
#endif
#ifndef CLAD3DGS_CTAS_PER_SM
#define CLAD3DGS_CTAS_PER_SM 2
#endif
constexpr int kTile = CLAD3DGS_TILE;              // Gaussians per tile
constexpr int kMaxCtasPerSm = CLAD3DGS_CTAS_PER_SM;  // cap on persistent CTAs per SM
constexpr int kConsumers = 512;                  // 16 warps: one per SH term
constexpr int kPersistThreads = kConsumers + 32;  // + 1 producer warp
constexpr int kMaxStages = 8;
constexpr int kUpdateFirst = 64;  // first consumer thread of phase B
static_assert(kTile == 32, "one lane per Gaussian of a tile");
// Dynamic shared memory for the stages of one CTA when `ctas` CTAs share an
// SM's 226 KB: less each CTA's static scratch and a reserve.
constexpr uint32_t stage_budget(int ctas) {
  return (226u * 1024u) / ctas -
         (16u * kTile * 3u + 48u * kTile + 2u * 14u * kTile) * 4u - 1536u;
}
constexpr uint32_t round_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

template <int Sh, bool Act, bool Snap, bool Xyz = false>
struct Cfg {
  static constexpr int kSh = Sh;
  static constexpr bool kAct = Act;
  static constexpr bool kSnap = Snap;
  // Torch-fused Adam on the positions too (dm is their complete gradient).
  static constexpr bool kXyz = Xyz && Sh == SH_SPLIT_TORCH;
  static constexpr bool written(int a) { return kWritten[a] || (kXyz && a == MEANS); }
  static constexpr bool has(int a) {
    if (a == XYZ_M || a == XYZ_V) return kXyz;
    if (a == MEANS || a == RADII || a == CLAMPED || a == SEED || a == DM)
      return Sh != SH_NONE;
    if (a == COEF) return Sh == SH_SGD || Sh == SH_ADAM;
    if (a == COEF_M || a == COEF_V) return Sh == SH_ADAM;
    if (a == DC || a == REST || a == DC_M || a == REST_M || a == DC_V || a == REST_V)
      return Sh == SH_SPLIT_ADAM || Sh == SH_SPLIT_TORCH;
    if (a == SNAP) return Snap && (Sh == SH_SPLIT_ADAM || Sh == SH_SPLIT_TORCH);
    return Act;  // activation parameters, moments, seeds, saved values
  }
  // Updated elements per Gaussian (parameters of every group, in region order).
  static constexpr int kDc = has(DC) ? 3 : 0, kRest = has(REST) ? 45 : 0,
                       kCoef = has(COEF) ? 48 : 0, kRot = Act ? 4 : 0,
                       kScl = Act ? 3 : 0, kOpa = Act ? 1 : 0;
  static constexpr int kParams = kDc + kRest + kCoef + kRot + kScl + kOpa;
  static constexpr uint32_t tile_bytes(int a) {
    return uint32_t(kTile) * kWidth[a] * elem_bytes(a);
  }
  static constexpr uint32_t offset(int a) {
    uint32_t o = 0;
    for (int b = 0; b < a; ++b)
      if (has(b)) o += round_up(tile_bytes(b), 128);
    return o;
  }
  static constexpr uint32_t stage_bytes = offset(NUM_ARR);
  static constexpr uint32_t load_bytes() {
    uint32_t s = 0;
    for (int a = 0; a < NUM_ARR; ++a)
      if (has(a)) s += tile_bytes(a);
    return s;
  }
  // As many CTAs per SM (up to the cap) as still get two stages each, then as
  // many stages per CTA as fit.
  static constexpr int ctas_fitting(int c) {
    return (c <= 1 || stage_budget(c) / stage_bytes >= 2) ? c : ctas_fitting(c - 1);
  }
  static constexpr int ctas = ctas_fitting(kMaxCtasPerSm);
  static constexpr int stages =
      (stage_budget(ctas) / stage_bytes) > kMaxStages
          ? kMaxStages
          : int(stage_budget(ctas) / stage_bytes);
  static_assert(stages >= 2, "stage does not fit twice in shared memory");
};

// Everything a launch needs; passed by value.
struct StepParams {
  const void* ptr[NUM_ARR];
  long long n;           // Gaussians
  long long tile_begin;  // first tile of this launch
  long long tile_end;    // one past the last tile of this launch
  const float* camera;   // device, 3 floats
  int degree;
  float sh_step_dc, sh_step_rest;            // torch Adam on dc / rest
  double sh_inv_bias2;                       // 1 / bias2_sqrt, rounded to double
  float inv_bias1, inv_bias2;                // float Adam (AdamConfig)
  float act_step[3];                         // rotation, scaling, opacity
  double act_inv_bias2[3];
  float xyz_step;                            // torch Adam on the positions
  double xyz_inv_bias2;
};

template <class F, int... Is>
__device__ __forceinline__ void for_each_arr_impl(F&& f,
                                                  std::integer_sequence<int, Is...>) {
  (f(std::integral_constant<int, Is>{}), ...);
}
template <class F>
__device__ __forceinline__ void for_each_arr(F&& f) {
  for_each_arr_impl(f, std::make_integer_sequence<int, NUM_ARR>{});
}

template <class C>
struct Stage {
  unsigned char* base;
  template <int A>
  __device__ __forceinline__ float* f() const {
    return reinterpret_cast<float*>(base + C::offset(A));
  }
  template <int A>
  __device__ __forceinline__ int* i() const {
    return reinterpret_cast<int*>(base + C::offset(A));
  }
  template <int A>
  __device__ __forceinline__ unsigned char* b() const {
    return base + C::offset(A);
  }
};

// ---------------------------------------------------------------------------
// Arithmetic on one staged tile (kTile Gaussians, 16 consumer warps).
//
// Phase A0: warp 0 (lane = Gaussian) computes each Gaussian's visibility, view
// direction and masked colour seed once; warps 1-3 compute the rotation /
// scaling / opacity VJPs meanwhile.
// Phase A1: warp j owns SH term j of every Gaussian of the tile (lane =
// Gaussian): it writes the coefficient gradient b_j * seed into a gradient tile
// laid out like the parameter region and the term's direction adjoint t_j into
// `partial`. The term index is warp-uniform and compile-time after a 16-way
// dispatch, so there is no divergent switch; rows of 45 (rest) or 3 (dc)
// floats are odd strides, so these accesses are bank-conflict free.
// Phase B: warp 0 finishes the position adjoint with the reference's
// shuffle-tree order ((t0+t8)+(t4+t12)) + ((t2+t10)+(t6+t14)) + ...
// (SHGradientConsumer.cu:203-207) while all consumers walk the parameter region
// (dc, rest, rotation, scaling, opacity share one index with the moments and
// the gradient tile) with one compact Adam update per element.

// Per-CTA scratch shared by the consumers. The per-Gaussian view data has two
// copies: warp 1 fills the next tile's while the current tile is updated.
struct __align__(16) Scratch {
  float partial[16][kTile][3];  // direction adjoint of every term
  __align__(16) float grad[kTile * 48];  // SH gradients, laid out like the parameters
  float dir[2][10][kTile];      // view direction of every Gaussian (x, y, z,
                                // r, xx, yy, zz, xy, yz, xz), one row per field
  float seed[2][kTile][3];      // clamped-masked colour seed
  int visible[2][kTile];
  int abort;                    // set by a consumer whose wait timed out
};

template <class C>
constexpr bool kSplit = C::kSh == SH_SPLIT_ADAM || C::kSh == SH_SPLIT_TORCH;

// Element offsets of each group inside the parameter (and gradient) region.
template <class C>
struct Region {
  static constexpr int kRest = kTile * C::kDc;
  static constexpr int kRot = kTile * (C::kDc + C::kRest + C::kCoef);
  static constexpr int kScl = kRot + kTile * C::kRot;
  static constexpr int kOpa = kScl + kTile * C::kScl;
  static constexpr int kTotal = kTile * C::kParams;
  static constexpr int first_of(int a0, int a1, int a2, int a3, int a4, int a5) {
    return C::has(a0) ? a0 : C::has(a1) ? a1 : C::has(a2) ? a2
         : C::has(a3) ? a3 : C::has(a4) ? a4 : a5;
  }
  static constexpr int kParamArr = first_of(DC, REST, COEF, ROT, SCL, OPA);
  static constexpr int kFirstArr = first_of(DC_M, REST_M, COEF_M, ROT_M, SCL_M, OPA_M);
  static constexpr int kSecondArr = first_of(DC_V, REST_V, COEF_V, ROT_V, SCL_V, OPA_V);
};

// Offset of term J, channel 0, of local Gaussian gl in the gradient tile.
template <class C, int J>
__device__ __forceinline__ int grad_offset(int gl) {
  if constexpr (kSplit<C>)
    return J == 0 ? gl * 3 : Region<C>::kRest + gl * 45 + 3 * (J - 1);
  else
    return gl * 48 + 3 * J;
}

template <class C, int J>
__device__ __forceinline__ const float* term_coefficients(const Stage<C>& st,
                                                          int gl) {
  if constexpr (!kSplit<C>) {
    return st.template f<COEF>() + gl * 48 + 3 * J;
  } else if constexpr (C::kSnap) {
    return st.template f<SNAP>() + gl * 48 + 3 * J;
  } else if constexpr (J == 0) {
    return st.template f<DC>() + gl * 3;
  } else {
    return st.template f<REST>() + gl * 45 + 3 * (J - 1);
  }
}

__device__ __forceinline__ void store_direction(Scratch& sc, int buf, int gl,
                                                const Direction& d) {
  const float f[10] = {d.x, d.y, d.z, d.r, d.xx, d.yy, d.zz, d.xy, d.yz, d.xz};
#pragma unroll
  for (int k = 0; k < 10; ++k) sc.dir[buf][k][gl] = f[k];
}

__device__ __forceinline__ Direction load_direction(const Scratch& sc, int buf, int gl) {
  const auto& r = sc.dir[buf];
  Direction d;
  d.x = r[0][gl]; d.y = r[1][gl]; d.z = r[2][gl];
  d.r = r[3][gl]; d.xx = r[4][gl]; d.yy = r[5][gl];
  d.zz = r[6][gl]; d.xy = r[7][gl]; d.yz = r[8][gl];
  d.xz = r[9][gl];
  return d;
}

// Phase A1 for term J of local Gaussian gl. Inactive terms (invisible
// Gaussian or above the degree) get a zero gradient, which still advances Adam.
template <class C, int J>
__device__ __forceinline__ void term_gradient(const Stage<C>& st, Scratch& sc,
                                              int buf, int gl, int nterms) {
  float* g = sc.grad + grad_offset<C, J>(gl);
  float* t = sc.partial[J][gl];
  if (sc.visible[buf][gl] && J < nterms) {
    const Direction d = load_direction(sc, buf, gl);
    const float* s = sc.seed[buf][gl];
    float b, gx, gy, gz;
    sh_basis<J>(d, b, gx, gy, gz);
    const float* c = term_coefficients<C, J>(st, gl);
    const float dot = (c[0] * s[0] + c[1] * s[1]) + c[2] * s[2];
    t[0] = gx * dot;
    t[1] = gy * dot;
    t[2] = gz * dot;
    g[0] = b * s[0];
    g[1] = b * s[1];
    g[2] = b * s[2];
  } else {
    t[0] = t[1] = t[2] = 0.f;
    g[0] = g[1] = g[2] = 0.f;
  }
}

// View data of a tile (one warp, lane = Gaussian): visibility, direction and
// clamp-masked colour seed into copy `buf` of the scratch.
template <class C>
__device__ __forceinline__ void phase_directions(const Stage<C>& st, Scratch& sc, int cnt,
                                                 int gl, const float cam[3], int buf) {
  if constexpr (C::kSh != SH_NONE) {
    if (gl >= cnt) return;
    const bool visible = st.template i<RADII>()[gl] > 0;
    sc.visible[buf][gl] = visible;
    if (visible) {
      const float* m = st.template f<MEANS>() + 3 * gl;
      store_direction(sc, buf, gl, make_direction(m[0], m[1], m[2], cam[0], cam[1], cam[2]));
      const unsigned char* cl = st.template b<CLAMPED>() + 3 * gl;
      const float* sd = st.template f<SEED>() + 3 * gl;
#pragma unroll
      for (int ch = 0; ch < 3; ++ch) sc.seed[buf][gl][ch] = cl[ch] ? 0.f : sd[ch];
    }
  }
}

// Activation VJPs for the float4 group at element e of the activation regions
// (controls/ManualActivations.cu:20-36, 94-100), computed in phase B: a rotation
// group is one Gaussian's quaternion (pv holds its values before the update);
// scaling and opacity groups are elementwise.
template <class C>
__device__ __forceinline__ float4 activation_gradient(const Stage<C>& st, int e,
                                                      const float4& pv) {
  using R = Region<C>;
  if (e < R::kScl) {
    const int gl = (e - R::kRot) >> 2;
    const float4 sq = *reinterpret_cast<const float4*>(st.template f<SEED_ROT>() + 4 * gl);
    const float qr[4] = {pv.x, pv.y, pv.z, pv.w};
    const float sr[4] = {sq.x, sq.y, sq.z, sq.w};
    float out[4];
    quaternion_vjp(qr, sr, st.template f<SAVED_NORM>()[gl], out);
    return make_float4(out[0], out[1], out[2], out[3]);
  }
  if (e < R::kOpa) {
    const int k = e - R::kScl;
    const float4 ss = *reinterpret_cast<const float4*>(st.template f<SEED_SCL>() + k);
    const float4 se = *reinterpret_cast<const float4*>(st.template f<SAVED_SCL>() + k);
    return make_float4(se.x * ss.x, se.y * ss.y, se.z * ss.z, se.w * ss.w);
  }
  const int k = e - R::kOpa;
  const float4 a = *reinterpret_cast<const float4*>(st.template f<SAVED_OPA>() + k);
  const float4 so = *reinterpret_cast<const float4*>(st.template f<SEED_OPA>() + k);
  return make_float4((a.x * (1.f - a.x)) * so.x, (a.y * (1.f - a.y)) * so.y,
                     (a.z * (1.f - a.z)) * so.z, (a.w * (1.f - a.w)) * so.w);
}

// Phase A1.
template <class C>
__device__ __forceinline__ void phase_terms(const StepParams& p,
                                            const Stage<C>& st, Scratch& sc,
                                            int cnt, int ct, int buf) {
  if constexpr (C::kSh != SH_NONE) {
    const int term = ct >> 5, gl = ct & 31;  // term is warp-uniform
    if (gl >= cnt) return;
    if (C::kSh == SH_SGD && !sc.visible[buf][gl]) return;  // SGD skips invisible
    const int nterms = (p.degree + 1) * (p.degree + 1);
    switch (term) {
      case 0: term_gradient<C, 0>(st, sc, buf, gl, nterms); break;
      case 1: term_gradient<C, 1>(st, sc, buf, gl, nterms); break;
      case 2: term_gradient<C, 2>(st, sc, buf, gl, nterms); break;
      case 3: term_gradient<C, 3>(st, sc, buf, gl, nterms); break;
      case 4: term_gradient<C, 4>(st, sc, buf, gl, nterms); break;
      case 5: term_gradient<C, 5>(st, sc, buf, gl, nterms); break;
      case 6: term_gradient<C, 6>(st, sc, buf, gl, nterms); break;
      case 7: term_gradient<C, 7>(st, sc, buf, gl, nterms); break;
      case 8: term_gradient<C, 8>(st, sc, buf, gl, nterms); break;
      case 9: term_gradient<C, 9>(st, sc, buf, gl, nterms); break;
      case 10: term_gradient<C, 10>(st, sc, buf, gl, nterms); break;
      case 11: term_gradient<C, 11>(st, sc, buf, gl, nterms); break;
      case 12: term_gradient<C, 12>(st, sc, buf, gl, nterms); break;
      case 13: term_gradient<C, 13>(st, sc, buf, gl, nterms); break;
      case 14: term_gradient<C, 14>(st, sc, buf, gl, nterms); break;
      default: term_gradient<C, 15>(st, sc, buf, gl, nterms); break;
    }
  }
}

// Position adjoint (warp 0, lane = Gaussian), after phase A: the direction
// adjoints of the 16 terms in the reference's tree order, into dm; then, in the
// configurations that own the positions, torch-fused Adam on them with dm as
// the gradient (every Gaussian, as the optimizer would).
template <class C>
__device__ __forceinline__ void finish_position(const StepParams& p, const Stage<C>& st,
                                                Scratch& sc, int cnt, int ct, int buf) {
  if constexpr (C::kSh != SH_NONE) {
    const int gl = ct & 31;
    if ((ct >> 5) != 0 || gl >= cnt) return;
    float* dm = st.template f<DM>() + 3 * gl;
    if (sc.visible[buf][gl]) {
      float dd[3];
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        float v[4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
          v[r] = (sc.partial[r][gl][k] + sc.partial[r + 8][gl][k]) +
                 (sc.partial[r + 4][gl][k] + sc.partial[r + 12][gl][k]);
        dd[k] = (v[0] + v[2]) + (v[1] + v[3]);
      }
      float o[3];
      direction_vjp(load_direction(sc, buf, gl), dd[0], dd[1], dd[2], o[0], o[1], o[2]);
#pragma unroll
      for (int k = 0; k < 3; ++k) dm[k] = dm[k] + o[k];
    }
    if constexpr (C::kXyz) {
      float* m = st.template f<MEANS>() + 3 * gl;
      float* first = st.template f<XYZ_M>() + 3 * gl;
      float* second = st.template f<XYZ_V>() + 3 * gl;
#pragma unroll
      for (int k = 0; k < 3; ++k)
        torch_adam(m[k], first[k], second[k], dm[k], p.xyz_step, p.xyz_inv_bias2);
    }
  }
}

// Phase B: one update per element of the parameter region. Slots past the
// tile's Gaussian count are updated too and never stored.
// Per-element updates of one float4 group; the group's region fixes the step
// size (every region is a multiple of four elements long).
template <class C>
__device__ __forceinline__ void update_group(const StepParams& p,
                                             const Stage<C>& st, int e,
                                             float4& pv, float4& mv, float4& vv,
                                             const float4& gv) {
  using R = Region<C>;
  if constexpr (C::kSh == SH_SPLIT_TORCH || C::kSh == SH_NONE) {
    float step = 0.f;
    double inv_bias2 = 1.0;
    if constexpr (C::kSh == SH_SPLIT_TORCH) {
      step = e < R::kRest ? p.sh_step_dc : p.sh_step_rest;
      inv_bias2 = p.sh_inv_bias2;
    }
    if constexpr (C::kAct) {
      if (C::kSh == SH_NONE || e >= R::kRot) {
        const int group = e < R::kScl ? 0 : (e < R::kOpa ? 1 : 2);
        step = p.act_step[group];
        inv_bias2 = p.act_inv_bias2[group];
      }
    }
    torch_adam(pv.x, mv.x, vv.x, gv.x, step, inv_bias2);
    torch_adam(pv.y, mv.y, vv.y, gv.y, step, inv_bias2);
    torch_adam(pv.z, mv.z, vv.z, gv.z, step, inv_bias2);
    torch_adam(pv.w, mv.w, vv.w, gv.w, step, inv_bias2);
  } else if constexpr (C::kSh == SH_SPLIT_ADAM) {
    const float rate = e < R::kRest ? kDcRate : kRestRate;
    float_adam(pv.x, mv.x, vv.x, gv.x, rate, p.inv_bias1, p.inv_bias2);
    float_adam(pv.y, mv.y, vv.y, gv.y, rate, p.inv_bias1, p.inv_bias2);
    float_adam(pv.z, mv.z, vv.z, gv.z, rate, p.inv_bias1, p.inv_bias2);
    float_adam(pv.w, mv.w, vv.w, gv.w, rate, p.inv_bias1, p.inv_bias2);
  } else if constexpr (C::kSh == SH_ADAM) {
    // Packed rows: term 0 (elements 0..2 of a Gaussian's 48) is dc.
    const int col = e % 48;
    float_adam(pv.x, mv.x, vv.x, gv.x, col < 3 ? kDcRate : kRestRate, p.inv_bias1, p.inv_bias2);
    float_adam(pv.y, mv.y, vv.y, gv.y, col + 1 < 3 ? kDcRate : kRestRate, p.inv_bias1, p.inv_bias2);
    float_adam(pv.z, mv.z, vv.z, gv.z, col + 2 < 3 ? kDcRate : kRestRate, p.inv_bias1, p.inv_bias2);
    float_adam(pv.w, mv.w, vv.w, gv.w, kRestRate, p.inv_bias1, p.inv_bias2);
  } else {
    // SGD leaves invisible Gaussians untouched (SHGradientConsumer.cu:93); the
    // four elements belong to one Gaussian (48 is a multiple of 4).
    if (st.template i<RADII>()[e / 48] > 0) {
      sgd(pv.x, gv.x);
      sgd(pv.y, gv.y);
      sgd(pv.z, gv.z);
      sgd(pv.w, gv.w);
    }
  }
}

// Each consumer of warps 2-15 updates four consecutive elements with 128-bit
// shared-memory accesses; every group's region is a multiple of four elements
// long, so the four share one group (one step size).
template <class C>
__device__ __forceinline__ void phase_update(const StepParams& p,
                                             const Stage<C>& st,
                                             const Scratch& sc, int ct) {
  using R = Region<C>;
  static_assert(R::kTotal % 4 == 0 && R::kRest % 4 == 0 && R::kRot % 4 == 0 &&
                    R::kScl % 4 == 0 && R::kOpa % 4 == 0,
                "group regions must be float4-aligned");
  constexpr bool kMoments = C::kSh != SH_SGD;
  float4* P = reinterpret_cast<float4*>(st.template f<R::kParamArr>());
  float4* M = kMoments ? reinterpret_cast<float4*>(st.template f<R::kFirstArr>()) : nullptr;
  float4* V = kMoments ? reinterpret_cast<float4*>(st.template f<R::kSecondArr>()) : nullptr;
  const float4* G = reinterpret_cast<const float4*>(sc.grad);
  // Warps 2-15 (448 threads: one float4 each for a full 56-parameter tile);
  // warp 0 is busy with the position adjoint meanwhile, and the tile's closing
  // barrier waits for the slowest warp.
  if (ct < kUpdateFirst) return;
  for (int q = ct - kUpdateFirst; q < R::kTotal / 4; q += kConsumers - kUpdateFirst) {
    const int e = 4 * q;
    const float4 pv0 = P[q];
    float4 pv = pv0, gv;
    if constexpr (C::kAct) {
      if (C::kSh == SH_NONE || e >= R::kRot) gv = activation_gradient<C>(st, e, pv0);
      else gv = G[q];
    } else {
      gv = G[q];
    }
    float4 mv = make_float4(0.f, 0.f, 0.f, 0.f), vv = mv;
    if constexpr (kMoments) {
      mv = M[q];
      vv = V[q];
    }
    update_group<C>(p, st, e, pv, mv, vv, gv);
    P[q] = pv;
    if constexpr (kMoments) {
      M[q] = mv;
      V[q] = vv;
    }
  }
}

// One whole tile (the one-tile kernel): warp 1 prepares the view data, then
// phase A, then the position adjoint (warp 0) and phase B (warps 2-15).
template <class C>
__device__ __forceinline__ void process_tile(const StepParams& p, const Stage<C>& st,
                                             Scratch& sc, int cnt, int ct,
                                             const float cam[3]) {
  if ((ct >> 5) == 1) phase_directions<C>(st, sc, cnt, ct & 31, cam, 0);
  named_barrier(1, kConsumers);
  phase_terms<C>(p, st, sc, cnt, ct, 0);
  named_barrier(1, kConsumers);
  finish_position<C>(p, st, sc, cnt, ct, 0);
  phase_update<C>(p, st, sc, ct);
}

template <class C>
__device__ __forceinline__ void load_camera(const StepParams& p, float cam[3]) {
  if constexpr (C::kSh != SH_NONE) {
    cam[0] = __ldg(p.camera);
    cam[1] = __ldg(p.camera + 1);
    cam[2] = __ldg(p.camera + 2);
  } else {
    cam[0] = cam[1] = cam[2] = 0.f;
  }
}

// Staging facts of array `lane` (one lane per array, NUM_ARR <= 32).
template <class C>
__device__ __forceinline__ void lane_array(int lane, bool& present, bool& written,
                                           uint32_t& offset, uint32_t& bytes) {
  present = written = false;
  offset = bytes = 0;
  for_each_arr([&](auto a_) {
    constexpr int a = decltype(a_)::value;
    if constexpr (C::has(a)) {
      constexpr bool kWrites = C::written(a);
      constexpr uint32_t kOffset = C::offset(a), kBytes = C::tile_bytes(a);
      if (lane == a) {
        present = true;
        written = kWrites;
        offset = kOffset;
        bytes = kBytes;
      }
    }
  });
}
static_assert(NUM_ARR <= 32, "one producer lane per staged array");

// ---------------------------------------------------------------------------
// Persistent pipeline: warp 0 produces (loads ahead, stores behind), the
// other warps consume.
template <class C>
__global__ void __launch_bounds__(kPersistThreads, C::ctas)
    stream_kernel(const StepParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full_bar[C::stages];
  __shared__ __align__(8) uint64_t done_bar[C::stages];
  __shared__ Scratch scratch;
  constexpr int S = C::stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&done_bar[s], 1);
    }
    scratch.abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const long long first = p.tile_begin + blockIdx.x;
  const long long stride = gridDim.x;

  if (warp == 0) {
    // Lane a loads and stores staged array a (one warp instruction per tile
    // for all arrays); lane 0 owns the barriers. Tile k goes to stage k % S.
    // Before the stage is reused for tile k + S, the producer waits until the
    // consumers have computed tile k, issues tile k's bulk stores and waits
    // until they have read the stage; the consumers never wait on a store.
    bool present, written;
    uint32_t off, bytes;
    lane_array<C>(lane, present, written, off, bytes);
    const char* base = present ? static_cast<const char*>(p.ptr[lane]) : nullptr;
    char* out = (present && written) ? static_cast<char*>(const_cast<void*>(p.ptr[lane]))
                                     : nullptr;
    auto drain = [&](int kd) -> bool {
      const int s = kd % S;
      int ok = 1;
      if (lane == 0) ok = mbar_wait_bounded(&done_bar[s], (kd / S) & 1) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) return false;
      if (out) {
        const long long t = first + (long long)kd * stride;
        bulk_store(out + t * (long long)bytes, smem + size_t(s) * C::stage_bytes + off, bytes);
        bulk_commit();
      }
      return true;
    };
    int k = 0;
    for (long long t = first; t < p.tile_end; t += stride, ++k) {
      const int s = k % S;
      if (k >= S) {
        if (!drain(k - S)) {
          if (lane == 0) atomicOr(&g_fault_word, kFaultProducerWait);
          bulk_wait_read<0>();
          return;
        }
        bulk_wait_read<0>();  // the stores of tile k - S have read stage s
        __syncwarp();
      }
      if (lane == 0) mbar_arrive_expect_tx(&full_bar[s], C::load_bytes());
      __syncwarp();
      if (present)
        bulk_load(smem + size_t(s) * C::stage_bytes + off, base + t * (long long)bytes,
                  bytes, &full_bar[s]);
    }
    for (int kd = k > S ? k - S : 0; kd < k; ++kd) {
      if (!drain(kd)) {
        if (lane == 0) atomicOr(&g_fault_word, kFaultProducerWait);
        break;
      }
    }
    bulk_wait_read<0>();
    return;
  }

  const int ct = threadIdx.x - 32;
  float cam[3];
  load_camera<C>(p, cam);
  // Warp 1 waits for each stage and fills that tile's view data one tile ahead
  // (the first before the loop, the next during phase B); the barrier that
  // follows its wait orders every other consumer after its acquire, so only
  // warp 1 waits on the full barriers.
  const int cw = ct >> 5;
  if (cw == 1 && first < p.tile_end) {
    if (!mbar_wait_bounded(&full_bar[0], 0)) {
      atomicOr(&g_fault_word, kFaultConsumerWait);
      scratch.abort = 1;
    } else {
      phase_directions<C>(Stage<C>{smem}, scratch, kTile, ct & 31, cam, 0);
    }
  }
  named_barrier(1, kConsumers);
  int k = 0;
  for (long long t = first; t < p.tile_end; t += stride, ++k) {
    if (scratch.abort) break;
    const int s = k % S, buf = k & 1;
    Stage<C> st{smem + size_t(s) * C::stage_bytes};
    phase_terms<C>(p, st, scratch, kTile, ct, buf);
    named_barrier(1, kConsumers);
    if (cw == 0) {
      finish_position<C>(p, st, scratch, kTile, ct, buf);
    } else if (cw == 1) {
      if (t + stride < p.tile_end) {
        const int k1 = k + 1, s1 = k1 % S;
        if (!mbar_wait_bounded(&full_bar[s1], (k1 / S) & 1)) {
          atomicOr(&g_fault_word, kFaultConsumerWait);
          scratch.abort = 1;
        } else {
          phase_directions<C>(Stage<C>{smem + size_t(s1) * C::stage_bytes}, scratch, kTile,
                              ct & 31, cam, k1 & 1);
        }
      }
    } else {
      phase_update<C>(p, st, scratch, ct);
    }
    fence_async_shared();
    named_barrier(1, kConsumers);
    if (ct == 0) mbar_arrive(&done_bar[s]);  // tile k computed: the producer stores it
  }
}

// ---------------------------------------------------------------------------
// One tile per CTA, plain loads and stores; any 4-byte alignment, any count.
template <class C>
__global__ void __launch_bounds__(kConsumers)
    tile_kernel(const StepParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ Scratch scratch;
  const long long tile = p.tile_begin + blockIdx.x;
  const long long g0 = tile * kTile;
  const int cnt = int(min((long long)kTile, p.n - g0));
  Stage<C> st{smem};
  if (threadIdx.x == 0) scratch.abort = 0;
  for_each_arr([&](auto a_) {
    constexpr int a = decltype(a_)::value;
    if constexpr (C::has(a)) {
      const int count = cnt * kWidth[a];
      const long long base = g0 * kWidth[a];
      if constexpr (a == CLAMPED) {
        const unsigned char* src = static_cast<const unsigned char*>(p.ptr[a]);
        for (int e = threadIdx.x; e < count; e += kConsumers)
          st.base[C::offset(a) + e] = src[base + e];
      } else {
        const float* src = static_cast<const float*>(p.ptr[a]);
        float* dst = reinterpret_cast<float*>(st.base + C::offset(a));
        for (int e = threadIdx.x; e < count; e += kConsumers)
          dst[e] = src[base + e];
      }
    }
  });
  float cam[3];
  load_camera<C>(p, cam);
  __syncthreads();
  process_tile<C>(p, st, scratch, cnt, threadIdx.x, cam);
  __syncthreads();
  for_each_arr([&](auto a_) {
    constexpr int a = decltype(a_)::value;
    if constexpr (C::has(a) && C::written(a)) {
      const int count = cnt * kWidth[a];
      const long long base = g0 * kWidth[a];
      float* dst = static_cast<float*>(const_cast<void*>(p.ptr[a]));
      const float* src = reinterpret_cast<const float*>(st.base + C::offset(a));
      for (int e = threadIdx.x; e < count; e += kConsumers)
        dst[base + e] = src[e];
    }
  });
}

// ---------------------------------------------------------------------------
// Standalone quaternion VJP: one thread per Gaussian, 16-byte rows.
template <bool Vec>
__global__ void quaternion_kernel(long long n, const float* __restrict__ q,
                                  const float* __restrict__ seed,
                                  const float* __restrict__ norms,
                                  float* __restrict__ out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float qv[4], sv[4], r[4];
    if constexpr (Vec) {
      const float4 a = reinterpret_cast<const float4*>(q)[i];
      const float4 b = reinterpret_cast<const float4*>(seed)[i];
      qv[0] = a.x; qv[1] = a.y; qv[2] = a.z; qv[3] = a.w;
      sv[0] = b.x; sv[1] = b.y; sv[2] = b.z; sv[3] = b.w;
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        qv[k] = q[4 * i + k];
        sv[k] = seed[4 * i + k];
      }
    }
    const float norm = norms[i];
    quaternion_vjp(qv, sv, norm, r);
    if constexpr (Vec) {
      reinterpret_cast<float4*>(out)[i] = make_float4(r[0], r[1], r[2], r[3]);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) out[4 * i + k] = r[k];
    }
  }
}

// ---------------------------------------------------------------------------
// Host side.

thread_local std::string t_last_error;

int fail(int code, const std::string& message) {
  t_last_error = message;
  return code;
}

struct DeviceInfo {
  int sm_count = 0;
};

DeviceInfo& device_info() {
  static DeviceInfo infos[64];
  int dev = 0;
  cudaGetDevice(&dev);
  DeviceInfo& info = infos[dev & 63];
  if (info.sm_count == 0) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    info.sm_count = sms > 0 ? sms : 1;
  }
  return info;
}

template <class C>
constexpr size_t persist_smem() { return size_t(C::stages) * C::stage_bytes; }

template <class C>
cudaError_t configure_kernels() {
  // Attributes are per function and cheap to set; setting them on every call
  // keeps multi-device processes correct without per-device bookkeeping.
  cudaError_t e = cudaFuncSetAttribute(stream_kernel<C>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(persist_smem<C>()));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(tile_kernel<C>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(C::stage_bytes));
}

template <class C>
cudaError_t run(StepParams p, cudaStream_t stream) {
  if (p.n <= 0) return cudaSuccess;
  cudaError_t e = configure_kernels<C>();
  if (e != cudaSuccess) return e;
  // Every array this configuration stages must be given; never launch with a
  // missing one.
  for (int a = 0; a < NUM_ARR; ++a)
    if (C::has(a) && p.ptr[a] == nullptr) return cudaErrorInvalidDevicePointer;
  if constexpr (C::kSh != SH_NONE)
    if (p.camera == nullptr) return cudaErrorInvalidDevicePointer;
  const long long tiles = (p.n + kTile - 1) / kTile;
  const long long full = p.n / kTile;
  bool aligned = true;
  for (int a = 0; a < NUM_ARR; ++a)
    if (C::has(a))
      aligned = aligned && (reinterpret_cast<uintptr_t>(p.ptr[a]) % 16 == 0);
  long long generic_begin = 0;
  if (aligned && full > 0) {
    const long long grid =
        std::min<long long>(full, (long long)device_info().sm_count * C::ctas);
    p.tile_begin = 0;
    p.tile_end = full;
    stream_kernel<C><<<unsigned(grid), kPersistThreads, persist_smem<C>(),
                       stream>>>(p);
    generic_begin = full;
  }
  if (generic_begin < tiles) {
    p.tile_begin = generic_begin;
    p.tile_end = tiles;
    tile_kernel<C><<<unsigned(tiles - generic_begin), kConsumers,
                     C::stage_bytes, stream>>>(p);
  }
  return cudaPeekAtLastError();
}

StepParams base_params(long long n) {
  StepParams p;
  std::memset(&p, 0, sizeof(p));
  p.n = n;
  return p;
}

void set_sh_inputs(StepParams& p, int degree, const float* means,
                   const int* radii, const bool* clamped, const float* camera,
                   const float* seed, float* dm) {
  p.degree = degree;
  p.ptr[MEANS] = means;
  p.ptr[RADII] = radii;
  p.ptr[CLAMPED] = clamped;
  p.ptr[SEED] = seed;
  p.ptr[DM] = dm;
  p.camera = camera;
}

void set_split(StepParams& p, const float* coefficient, float* dc, float* rest,
               float* dc_first, float* dc_second, float* rest_first,
               float* rest_second) {
  p.ptr[SNAP] = coefficient;
  p.ptr[DC] = dc;
  p.ptr[DC_M] = dc_first;
  p.ptr[DC_V] = dc_second;
  p.ptr[REST] = rest;
  p.ptr[REST_M] = rest_first;
  p.ptr[REST_V] = rest_second;
}

void set_torch_config(StepParams& p, TorchAdamConfig c) {
  // rate / bias1 in double, rounded once to float, as torch fused Adam does.
  p.sh_step_dc = float(0.0025 / double(c.bias1));
  p.sh_step_rest = float(0.000125 / double(c.bias1));
  p.sh_inv_bias2 = 1.0 / double(c.bias2_sqrt);
}

void set_activations(StepParams& p, float* const* parameters,
                     const float* const* seeds, const float* const* saved,
                     float* const* first, float* const* second,
                     const double* rates, const float* bias1,
                     const float* bias2) {
  constexpr int kParam[3] = {ROT, SCL, OPA};
  constexpr int kFirst[3] = {ROT_M, SCL_M, OPA_M};
  constexpr int kSecond[3] = {ROT_V, SCL_V, OPA_V};
  constexpr int kSeed[3] = {SEED_ROT, SEED_SCL, SEED_OPA};
  constexpr int kSaved[3] = {SAVED_NORM, SAVED_SCL, SAVED_OPA};
  for (int j = 0; j < 3; ++j) {
    p.ptr[kParam[j]] = parameters[j];
    p.ptr[kFirst[j]] = first[j];
    p.ptr[kSecond[j]] = second[j];
    p.ptr[kSeed[j]] = seeds[j];
    p.ptr[kSaved[j]] = saved[j];
    p.act_step[j] = float(rates[j] / double(bias1[j]));
    p.act_inv_bias2[j] = 1.0 / double(bias2[j]);
  }
}

void set_xyz(StepParams& p, float* first, float* second, double rate, TorchAdamConfig c) {
  p.ptr[XYZ_M] = first;
  p.ptr[XYZ_V] = second;
  p.xyz_step = float(rate / double(c.bias1));
  p.xyz_inv_bias2 = 1.0 / double(c.bias2_sqrt);
}

bool degree_ok(int degree) { return degree >= 0 && degree <= 3; }

int status_of(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return CLAD3DGS_OK;
  cudaGetLastError();  // clear a non-sticky launch error for the next call
  return fail(CLAD3DGS_CUDA_ERROR, std::string(what) + ": " + cudaGetErrorString(e));
}

using SplitTorch = Cfg<SH_SPLIT_TORCH, false, false>;
using SplitTorchSnap = Cfg<SH_SPLIT_TORCH, false, true>;
using SplitAdam = Cfg<SH_SPLIT_ADAM, false, false>;
using SplitAdamSnap = Cfg<SH_SPLIT_ADAM, false, true>;
using PackedAdam = Cfg<SH_ADAM, false, false>;
using PackedSgd = Cfg<SH_SGD, false, false>;
using ActOnly = Cfg<SH_NONE, true, false>;
using Fused = Cfg<SH_SPLIT_TORCH, true, false>;
using FusedSnap = Cfg<SH_SPLIT_TORCH, true, true>;
using SplitTorchXyz = Cfg<SH_SPLIT_TORCH, false, false, true>;
using SplitTorchXyzSnap = Cfg<SH_SPLIT_TORCH, false, true, true>;
using FusedXyz = Cfg<SH_SPLIT_TORCH, true, false, true>;
using FusedXyzSnap = Cfg<SH_SPLIT_TORCH, true, true, true>;

cudaError_t run_split_torch(StepParams& p, cudaStream_t stream) {
  return p.ptr[SNAP] ? run<SplitTorchSnap>(p, stream) : run<SplitTorch>(p, stream);
}

cudaError_t launch_quaternion(long long n, const float* q, const float* seed,
                              const float* norms, float* out,
                              cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const bool vec = (reinterpret_cast<uintptr_t>(q) |
                    reinterpret_cast<uintptr_t>(seed) |
                    reinterpret_cast<uintptr_t>(out)) % 16 == 0;
  const long long blocks = std::min<long long>(
      (n + 255) / 256, (long long)device_info().sm_count * 16);
  if (vec)
    quaternion_kernel<true><<<unsigned(blocks), 256, 0, stream>>>(n, q, seed,
                                                                  norms, out);
  else
    quaternion_kernel<false><<<unsigned(blocks), 256, 0, stream>>>(n, q, seed,
                                                                   norms, out);
  return cudaPeekAtLastError();
}

}  // namespace clad3dgs

using namespace clad3dgs;

// ===================== drop-in entries =====================

extern "C" void sh_consumer_sgd(int n, int degree, const float* means,
                                const int* radii, float* coeff,
                                const bool* clamped, const float* camera,
                                const float* seed, float* dm) {
  if (n <= 0) return;
  if (!degree_ok(degree))
    throw std::invalid_argument("SH degree must be between zero and three");
  StepParams p = base_params(n);
  set_sh_inputs(p, degree, means, radii, clamped, camera, seed, dm);
  p.ptr[COEF] = coeff;
  run<PackedSgd>(p, 0);
}

extern "C" void sh_consumer_adam(int n, int degree, const float* means,
                                 const int* radii, float* coeff,
                                 const bool* clamped, const float* camera,
                                 const float* seed, float* dm, float* first,
                                 float* second, AdamConfig config) {
  if (n <= 0) return;
  if (!degree_ok(degree))
    throw std::invalid_argument("SH degree must be between zero and three");
  StepParams p = base_params(n);
  set_sh_inputs(p, degree, means, radii, clamped, camera, seed, dm);
  p.ptr[COEF] = coeff;
  p.ptr[COEF_M] = first;
  p.ptr[COEF_V] = second;
  p.inv_bias1 = config.inv_bias1;
  p.inv_bias2 = config.inv_bias2;
  run<PackedAdam>(p, 0);
}

extern "C" void sh_consumer_split_adam(int n, int degree, const float* means,
                                       const int* radii,
                                       const float* coefficient,
                                       const bool* clamped, const float* camera,
                                       const float* seed, float* dm, float* dc,
                                       float* rest, float* dc_first,
                                       float* dc_second, float* rest_first,
                                       float* rest_second, AdamConfig config) {
  if (n <= 0) return;
  if (!degree_ok(degree))
    throw std::invalid_argument("SH degree must be between zero and three");
  StepParams p = base_params(n);
  set_sh_inputs(p, degree, means, radii, clamped, camera, seed, dm);
  set_split(p, coefficient, dc, rest, dc_first, dc_second, rest_first,
            rest_second);
  p.inv_bias1 = config.inv_bias1;
  p.inv_bias2 = config.inv_bias2;
  if (coefficient)
    run<SplitAdamSnap>(p, 0);
  else
    run<SplitAdam>(p, 0);
}

extern "C" void sh_consumer_split_torch_adam(
    int n, int degree, const float* means, const int* radii,
    const float* coefficient, const bool* clamped, const float* camera,
    const float* seed, float* dm, float* dc, float* rest, float* dc_first,
    float* dc_second, float* rest_first, float* rest_second,
    TorchAdamConfig config) {
  if (n <= 0) return;
  if (!degree_ok(degree))
    throw std::invalid_argument("SH degree must be between zero and three");
  StepParams p = base_params(n);
  set_sh_inputs(p, degree, means, radii, clamped, camera, seed, dm);
  set_split(p, coefficient, dc, rest, dc_first, dc_second, rest_first,
            rest_second);
  set_torch_config(p, config);
  run_split_torch(p, 0);
}

extern "C" void launch_activation_consume(int n, float* const* parameters,
                                          const float* const* seeds,
                                          const float* const* saved,
                                          float* const* first,
                                          float* const* second,
                                          const double* rates,
                                          const float* bias1, const float* bias2,
                                          cudaStream_t stream) {
  if (n <= 0) return;
  StepParams p = base_params(n);
  set_activations(p, parameters, seeds, saved, first, second, rates, bias1,
                  bias2);
  run<ActOnly>(p, stream);
}

extern "C" void launch_quaternion_backward(int n, const float* q,
                                           const float* seed,
                                           const float* norms, float* out,
                                           cudaStream_t stream) {
  launch_quaternion(n, q, seed, norms, out, stream);
}

// ===================== clad3dgs_* entries =====================

extern "C" const char* clad3dgs_last_error(void) { return t_last_error.c_str(); }

extern "C" int clad3dgs_describe(int* sm_count, int* tile_gaussians,
                                 int* sh_stages, int* fused_stages) {
  if (sm_count) *sm_count = device_info().sm_count;
  if (tile_gaussians) *tile_gaussians = kTile;
  if (sh_stages) *sh_stages = SplitTorch::stages;
  if (fused_stages) *fused_stages = Fused::stages;
  return CLAD3DGS_OK;
}

extern "C" int clad3dgs_fault_status(int clear, unsigned int* fault_word) {
  unsigned int word = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&word, g_fault_word, sizeof(word));
  if (e != cudaSuccess) return status_of(e, "reading the fault word");
  if (clear && word) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_fault_word, &zero, sizeof(zero));
    if (e != cudaSuccess) return status_of(e, "clearing the fault word");
  }
  if (fault_word) *fault_word = word;
  return word ? fail(CLAD3DGS_DEVICE_FAULT, "a pipeline wait timed out")
              : CLAD3DGS_OK;
}

extern "C" int clad3dgs_sh_consume_split_torch_adam(
    int64_t n, int degree, const float* means, const int* radii,
    const float* coefficient, const bool* clamped, const float* camera,
    const float* seed, float* dm, float* dc, float* rest, float* dc_first,
    float* dc_second, float* rest_first, float* rest_second,
    TorchAdamConfig config, cudaStream_t stream) {
  if (n <= 0) return CLAD3DGS_OK;
  if (!degree_ok(degree))
    return fail(CLAD3DGS_INVALID_ARGUMENT,
                "SH degree must be between zero and three");
  StepParams p = base_params(n);
  set_sh_inputs(p, degree, means, radii, clamped, camera, seed, dm);
  set_split(p, coefficient, dc, rest, dc_first, dc_second, rest_first,
            rest_second);
  set_torch_config(p, config);
  return status_of(run_split_torch(p, stream), "SH consume launch");
}

extern "C" int clad3dgs_sh_consume_variant(
    int mode, int64_t n, int degree, const float* means, const int* radii,
    const float* coefficient, const bool* clamped, const float* camera,
    const float* seed, float* dm, float* coeff, float* first, float* second,
    float* dc, float* rest, float* dc_first, float* dc_second,
    float* rest_first, float* rest_second, AdamConfig config,
    cudaStream_t stream) {
  if (mode < 0 || mode > 2)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "unknown SH update mode");
  if (n <= 0) return CLAD3DGS_OK;
  if (!degree_ok(degree))
    return fail(CLAD3DGS_INVALID_ARGUMENT,
                "SH degree must be between zero and three");
  StepParams p = base_params(n);
  set_sh_inputs(p, degree, means, radii, clamped, camera, seed, dm);
  p.inv_bias1 = config.inv_bias1;
  p.inv_bias2 = config.inv_bias2;
  cudaError_t e;
  if (mode == 0) {
    p.ptr[COEF] = coeff;
    e = run<PackedSgd>(p, stream);
  } else if (mode == 1) {
    p.ptr[COEF] = coeff;
    p.ptr[COEF_M] = first;
    p.ptr[COEF_V] = second;
    e = run<PackedAdam>(p, stream);
  } else {
    set_split(p, coefficient, dc, rest, dc_first, dc_second, rest_first,
              rest_second);
    e = coefficient ? run<SplitAdamSnap>(p, stream) : run<SplitAdam>(p, stream);
  }
  return status_of(e, "SH consume launch");
}

extern "C" int clad3dgs_activation_consume(int64_t n, float* const* parameters,
                                           const float* const* seeds,
                                           const float* const* saved,
                                           float* const* first,
                                           float* const* second,
                                           const double* rates,
                                           const float* bias1,
                                           const float* bias2,
                                           cudaStream_t stream) {
  if (n <= 0) return CLAD3DGS_OK;
  StepParams p = base_params(n);
  set_activations(p, parameters, seeds, saved, first, second, rates, bias1,
                  bias2);
  return status_of(run<ActOnly>(p, stream), "activation consume launch");
}

extern "C" int clad3dgs_quaternion_backward(int64_t n, const float* q,
                                            const float* seed,
                                            const float* norms, float* out,
                                            cudaStream_t stream) {
  return status_of(launch_quaternion(n, q, seed, norms, out, stream),
                   "quaternion backward launch");
}

extern "C" int clad3dgs_gaussian_step(
    int64_t n, int degree, const float* means, const int* radii,
    const float* coefficient, const bool* clamped, const float* camera,
    const float* seed, float* dm, float* dc, float* rest, float* dc_first,
    float* dc_second, float* rest_first, float* rest_second,
    TorchAdamConfig sh_config, float* const* parameters,
    const float* const* seeds, const float* const* saved, float* const* first,
    float* const* second, const double* rates, const float* bias1,
    const float* bias2, cudaStream_t stream) {
  if (n <= 0) return CLAD3DGS_OK;
  if (!degree_ok(degree))
    return fail(CLAD3DGS_INVALID_ARGUMENT,
                "SH degree must be between zero and three");
  StepParams p = base_params(n);
  set_sh_inputs(p, degree, means, radii, clamped, camera, seed, dm);
  set_split(p, coefficient, dc, rest, dc_first, dc_second, rest_first,
            rest_second);
  set_torch_config(p, sh_config);
  set_activations(p, parameters, seeds, saved, first, second, rates, bias1,
                  bias2);
  cudaError_t e = coefficient ? run<FusedSnap>(p, stream) : run<Fused>(p, stream);
  return status_of(e, "fused Gaussian step launch");
}

extern "C" int clad3dgs_sh_consume_xyz(
    int64_t n, int degree, float* means, const int* radii, const float* coefficient,
    const bool* clamped, const float* camera, const float* seed, float* dm, float* dc,
    float* rest, float* dc_first, float* dc_second, float* rest_first, float* rest_second,
    TorchAdamConfig sh_config, float* xyz_first, float* xyz_second, double xyz_rate,
    TorchAdamConfig xyz_config, cudaStream_t stream) {
  if (n <= 0) return CLAD3DGS_OK;
  if (!degree_ok(degree))
    return fail(CLAD3DGS_INVALID_ARGUMENT,
                "SH degree must be between zero and three");
  StepParams p = base_params(n);
  set_sh_inputs(p, degree, means, radii, clamped, camera, seed, dm);
  set_split(p, coefficient, dc, rest, dc_first, dc_second, rest_first,
            rest_second);
  set_torch_config(p, sh_config);
  set_xyz(p, xyz_first, xyz_second, xyz_rate, xyz_config);
  cudaError_t e = coefficient ? run<SplitTorchXyzSnap>(p, stream)
                              : run<SplitTorchXyz>(p, stream);
  return status_of(e, "SH + position consume launch");
}

extern "C" int clad3dgs_gaussian_step_xyz(
    int64_t n, int degree, float* means, const int* radii, const float* coefficient,
    const bool* clamped, const float* camera, const float* seed, float* dm, float* dc,
    float* rest, float* dc_first, float* dc_second, float* rest_first, float* rest_second,
    TorchAdamConfig sh_config, float* const* parameters, const float* const* seeds,
    const float* const* saved, float* const* first, float* const* second,
    const double* rates, const float* bias1, const float* bias2, float* xyz_first,
    float* xyz_second, double xyz_rate, TorchAdamConfig xyz_config, cudaStream_t stream) {
  if (n <= 0) return CLAD3DGS_OK;
  if (!degree_ok(degree))
    return fail(CLAD3DGS_INVALID_ARGUMENT,
                "SH degree must be between zero and three");
  StepParams p = base_params(n);
  set_sh_inputs(p, degree, means, radii, clamped, camera, seed, dm);
  set_split(p, coefficient, dc, rest, dc_first, dc_second, rest_first,
            rest_second);
  set_torch_config(p, sh_config);
  set_activations(p, parameters, seeds, saved, first, second, rates, bias1,
                  bias2);
  set_xyz(p, xyz_first, xyz_second, xyz_rate, xyz_config);
  cudaError_t e = coefficient ? run<FusedXyzSnap>(p, stream) : run<FusedXyz>(p, stream);
  return status_of(e, "fused Gaussian step launch");
}
