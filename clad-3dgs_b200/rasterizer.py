"""The Gaussian-rasterizer extension surface over the C ABI.

The reference injects its renderer module as `diff_gaussian_rasterization._C`
(run.py:60-62) and calls it from adapter.py:21-117 and check.py:743-1052. This
module provides the same functions with the same argument order, meaning and
results, backed by libclad3dgs_b200.so:

* `rasterize_gaussians(bg, means3D, colors, opacity, scales, rotations,
  scale_modifier, cov3D_precomp, viewmatrix, projmatrix, tanfovx, tanfovy,
  image_height, image_width, sh, degree, campos, prefiltered, antialiasing,
  debug) -> (num_rendered, color, radii, geomBuffer, binningBuffer, imgBuffer,
  invdepths)`
* `rasterize_gaussians_backward(bg, means3D, radii, colors, opacities, scales,
  rotations, scale_modifier, cov3D_precomp, viewmatrix, projmatrix, tanfovx,
  tanfovy, dL_dout_color, dL_dout_invdepth, sh, degree, campos, geomBuffer, R,
  binningBuffer, imageBuffer, antialiasing, debug) -> (dL_dmeans2D, dL_dcolors,
  dL_dopacity, dL_dmeans3D, dL_dcov3D, dL_dsh, dL_dscales, dL_drotations)`
* `rasterize_gaussians_backward_consume(<the 24 above>, dc, rest, dc_first,
  dc_second, rest_first, rest_second, bias1, bias2_sqrt, *, xyz=None)`: the SH
  adjoint goes to the fused SH + Adam kernel (dc/rest and moments updated in
  place) and the returned dL_dsh is empty (prepare_native.py:32-93). With
  `xyz={first, second, rate, bias1, bias2_sqrt}` the same kernel also runs the
  positions' Adam (means3D updated in place; an addition of this package).
* `*_direct` variants take (dc, rest) in place of the packed `sh`
  (direct_inputs.py:80-220).
* `mark_visible(means3D, viewmatrix, projmatrix)`.

Also `GaussianRasterizationSettings` and `GaussianRasterizer`, the autograd
front end the trainer uses on steps that are not consumed.

`pixel_accumulation` selects the pixel-backward accumulation: 2 (default,
converged warps with a transposing reduction), 1 (the reference's full-warp
helper) or 0 (per-lane atomics).
"""

from __future__ import annotations

import ctypes
from typing import NamedTuple

import torch

import _native as native

pixel_accumulation = 2
MAX_SH_COEFFS = 16


def _check(condition, message):
    if not condition:
        raise RuntimeError(message)


class _Buffers:
    """Owns the torch tensors the C ABI requests through its allocation callback."""

    def __init__(self, device):
        self.device = device
        self.tensors = {0: None, 1: None, 2: None}

        def allocate(_ctx, which, nbytes):
            t = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=self.device)
            self.tensors[int(which)] = t
            return t.data_ptr()

        self.callback = native.ALLOC_FN(allocate)

    def get(self, which):
        t = self.tensors[which]
        return t if t is not None else torch.empty(0, dtype=torch.uint8, device=self.device)


def _contig(t):
    return None if t is None or t.numel() == 0 else t.contiguous()


def _sh_args(sh=None, dc=None, rest=None):
    if sh is not None and sh.numel():
        _check(sh.dim() == 3 and sh.shape[1] == MAX_SH_COEFFS and sh.shape[2] == 3,
               "SH coefficients must be [P, 16, 3]")
        return sh.contiguous(), None, None
    if dc is not None:
        return None, dc.contiguous(), rest.contiguous()
    return None, None, None


def _forward(bg, means3D, colors, opacity, scales, rotations, scale_modifier, cov3D_precomp,
             viewmatrix, projmatrix, tanfovx, tanfovy, image_height, image_width, sh_packed,
             dc, rest, degree, campos, antialiasing):
    device = means3D.device
    P = means3D.shape[0]
    _check(means3D.is_cuda and means3D.dim() == 2 and means3D.shape[1] == 3,
           "means3D must have dimensions (num_points, 3)")
    H, W = int(image_height), int(image_width)
    out_color = torch.empty((3, H, W), dtype=torch.float32, device=device)
    out_invdepth = torch.empty((1, H, W), dtype=torch.float32, device=device)
    radii = torch.zeros((P,), dtype=torch.int32, device=device)
    buffers = _Buffers(device)
    num_rendered = ctypes.c_int(0)
    tensors = dict(bg=bg.contiguous(), means=means3D.contiguous(), colors=_contig(colors),
                   opacity=opacity.contiguous(), scales=_contig(scales),
                   rotations=_contig(rotations), cov=_contig(cov3D_precomp),
                   view=viewmatrix.contiguous(), proj=projmatrix.contiguous(),
                   campos=campos.contiguous(), sh=sh_packed, dc=dc, rest=rest)
    status = native.library().clad3dgs_raster_forward(
        P, int(degree), native.ptr(tensors["bg"]), native.ptr(tensors["means"]),
        native.ptr(tensors["colors"]), native.ptr(tensors["opacity"]),
        native.ptr(tensors["scales"]), float(scale_modifier), native.ptr(tensors["rotations"]),
        native.ptr(tensors["cov"]), native.ptr(tensors["view"]), native.ptr(tensors["proj"]),
        float(tanfovx), float(tanfovy), H, W, native.ptr(tensors["sh"]),
        native.ptr(tensors["dc"]), native.ptr(tensors["rest"]), native.ptr(tensors["campos"]),
        int(bool(antialiasing)), ctypes.cast(buffers.callback, ctypes.c_void_p), None,
        out_color.data_ptr(), out_invdepth.data_ptr(), radii.data_ptr(),
        ctypes.byref(num_rendered), native.stream_handle())
    native.check(status, "rasterize_gaussians")
    return (num_rendered.value, out_color, radii, buffers.get(0), buffers.get(2),
            buffers.get(1), out_invdepth)


def rasterize_gaussians(bg, means3D, colors, opacity, scales, rotations, scale_modifier,
                        cov3D_precomp, viewmatrix, projmatrix, tanfovx, tanfovy,
                        image_height, image_width, sh, degree, campos, prefiltered,
                        antialiasing, debug):
    sh_packed, _, _ = _sh_args(sh)
    return _forward(bg, means3D, colors, opacity, scales, rotations, scale_modifier,
                    cov3D_precomp, viewmatrix, projmatrix, tanfovx, tanfovy, image_height,
                    image_width, sh_packed, None, None, degree, campos, antialiasing)


def rasterize_gaussians_direct(bg, means3D, colors, opacity, scales, rotations,
                               scale_modifier, cov3D_precomp, viewmatrix, projmatrix, tanfovx,
                               tanfovy, image_height, image_width, dc, rest, degree, campos,
                               prefiltered, antialiasing, debug):
    _check_direct(means3D, dc, rest, degree)
    return _forward(bg, means3D, colors, opacity, scales, rotations, scale_modifier,
                    cov3D_precomp, viewmatrix, projmatrix, tanfovx, tanfovy, image_height,
                    image_width, None, dc.contiguous(), rest.contiguous(), degree, campos,
                    antialiasing)


def _check_direct(means3D, dc, rest, degree):
    # direct_inputs.py:331-344
    n = means3D.shape[0]
    _check(0 <= degree <= 3 and tuple(dc.shape) == (n, 1, 3) and tuple(rest.shape) == (n, 15, 3),
           "unsupported direct SH layout")
    for t in (dc, rest):
        _check(t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()
               and t.device == means3D.device,
               "direct SH tensors must be contiguous CUDA float32 on the renderer device")
    _check_disjoint([dc, rest], "direct SH coefficient and moment buffers must be disjoint")


def _check_disjoint(tensors, message):
    spans = sorted((t.data_ptr(), t.data_ptr() + t.numel() * t.element_size())
                   for t in tensors if t.numel())
    _check(all(a[1] <= b[0] for a, b in zip(spans, spans[1:])), message)


def _backward(bg, means3D, radii, colors, opacities, scales, rotations, scale_modifier,
              cov3D_precomp, viewmatrix, projmatrix, tanfovx, tanfovy, dL_dout_color,
              dL_dout_invdepth, sh_packed, dc, rest, degree, campos, geomBuffer, R,
              binningBuffer, imageBuffer, antialiasing, consume=None):
    device = means3D.device
    P = means3D.shape[0]
    H, W = dL_dout_color.shape[1], dL_dout_color.shape[2]
    M = MAX_SH_COEFFS if (sh_packed is not None or dc is not None) else 0
    z = lambda *shape: torch.zeros(shape, dtype=torch.float32, device=device)
    g = dict(mean2d=z(P, 3), colors=z(P, 3), opacity=z(P, 1), means=z(P, 3), cov=z(P, 6),
             sh=z(P, M, 3) if consume is None else torch.empty(0, device=device),
             scales=z(P, 3), rotations=z(P, 4), conic=z(P, 4), invdepth=z(P, 1))
    if P == 0:
        return (g["mean2d"], g["colors"], g["opacity"], g["means"], g["cov"], g["sh"],
                g["scales"], g["rotations"])
    c = consume or {}
    b1, b2 = (consume["bias1"], consume["bias2_sqrt"]) if consume else (1.0, 1.0)
    xyz = c.get("xyz") or {}
    dpix = dL_dout_color.contiguous()
    dinv = _contig(dL_dout_invdepth)
    keep = dict(bg=bg.contiguous(), means=means3D.contiguous(), radii=radii.contiguous(),
                colors=_contig(colors), op=opacities.contiguous(), scales=_contig(scales),
                rot=_contig(rotations), cov=_contig(cov3D_precomp), view=viewmatrix.contiguous(),
                proj=projmatrix.contiguous(), campos=campos.contiguous())
    status = native.library().clad3dgs_raster_backward(
        P, int(degree), native.ptr(keep["bg"]), native.ptr(keep["means"]),
        native.ptr(keep["radii"]), native.ptr(keep["colors"]), native.ptr(keep["op"]),
        native.ptr(keep["scales"]), float(scale_modifier), native.ptr(keep["rot"]),
        native.ptr(keep["cov"]), native.ptr(keep["view"]), native.ptr(keep["proj"]),
        float(tanfovx), float(tanfovy), H, W, dpix.data_ptr(), native.ptr(dinv),
        native.ptr(sh_packed), native.ptr(dc), native.ptr(rest), native.ptr(keep["campos"]),
        native.ptr(geomBuffer), int(R), native.ptr(binningBuffer), native.ptr(imageBuffer),
        int(bool(antialiasing)), g["mean2d"].data_ptr(), g["colors"].data_ptr(),
        g["opacity"].data_ptr(), g["means"].data_ptr(), g["cov"].data_ptr(),
        native.ptr(g["sh"]), g["scales"].data_ptr(), g["rotations"].data_ptr(),
        g["conic"].data_ptr(), g["invdepth"].data_ptr(), int(pixel_accumulation),
        int(consume is not None), native.ptr(c.get("dc")), native.ptr(c.get("rest")),
        native.ptr(c.get("dc_first")), native.ptr(c.get("dc_second")),
        native.ptr(c.get("rest_first")), native.ptr(c.get("rest_second")),
        native.TorchAdamConfig(b1, b2), native.ptr(xyz.get("first")),
        native.ptr(xyz.get("second")), float(xyz.get("rate", 0.0)),
        native.TorchAdamConfig(xyz.get("bias1", 1.0), xyz.get("bias2_sqrt", 1.0)),
        native.stream_handle())
    native.check(status, "rasterize_gaussians_backward")
    return (g["mean2d"], g["colors"], g["opacity"], g["means"], g["cov"], g["sh"],
            g["scales"], g["rotations"])


def rasterize_gaussians_backward(bg, means3D, radii, colors, opacities, scales, rotations,
                                 scale_modifier, cov3D_precomp, viewmatrix, projmatrix,
                                 tanfovx, tanfovy, dL_dout_color, dL_dout_invdepth, sh, degree,
                                 campos, geomBuffer, R, binningBuffer, imageBuffer,
                                 antialiasing, debug):
    sh_packed, _, _ = _sh_args(sh)
    return _backward(bg, means3D, radii, colors, opacities, scales, rotations, scale_modifier,
                     cov3D_precomp, viewmatrix, projmatrix, tanfovx, tanfovy, dL_dout_color,
                     dL_dout_invdepth, sh_packed, None, None, degree, campos, geomBuffer, R,
                     binningBuffer, imageBuffer, antialiasing)


def rasterize_gaussians_backward_direct(bg, means3D, radii, colors, opacities, scales,
                                        rotations, scale_modifier, cov3D_precomp, viewmatrix,
                                        projmatrix, tanfovx, tanfovy, dL_dout_color,
                                        dL_dout_invdepth, dc, rest, degree, campos, geomBuffer,
                                        R, binningBuffer, imageBuffer, antialiasing, debug):
    _check_direct(means3D, dc, rest, degree)
    return _backward(bg, means3D, radii, colors, opacities, scales, rotations, scale_modifier,
                     cov3D_precomp, viewmatrix, projmatrix, tanfovx, tanfovy, dL_dout_color,
                     dL_dout_invdepth, None, dc.contiguous(), rest.contiguous(), degree,
                     campos, geomBuffer, R, binningBuffer, imageBuffer, antialiasing)


def _consume_state(means3D, degree, dc, rest, dc_first, dc_second, rest_first, rest_second,
                   bias1, bias2_sqrt, xyz=None):
    # prepare_native.py:52-67: default stream, split shapes and layouts.
    _check(torch.cuda.current_stream().cuda_stream == 0,
           "SH consumption requires the default CUDA stream")
    P = means3D.shape[0]
    _check(0 <= degree <= 3, "unsupported SH layout")
    for t in (dc, rest, dc_first, dc_second, rest_first, rest_second):
        _check(t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()
               and t.device == means3D.device,
               "split coefficient/moment tensors must be contiguous CUDA float32 on the "
               "renderer device")
    _check(dc.numel() == 3 * P and dc_first.numel() == 3 * P and dc_second.numel() == 3 * P
           and rest.numel() == 45 * P and rest_first.numel() == 45 * P
           and rest_second.numel() == 45 * P, "bad split coefficient or optimizer-state shape")
    state = dict(dc=dc, rest=rest, dc_first=dc_first, dc_second=dc_second,
                 rest_first=rest_first, rest_second=rest_second, bias1=float(bias1),
                 bias2_sqrt=float(bias2_sqrt))
    if xyz is not None:
        # The positions' Adam in the same kernel: means3D is updated in place.
        for t in (means3D, xyz["first"], xyz["second"]):
            _check(t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()
                   and t.device == means3D.device and t.numel() == 3 * P,
                   "positions and their moments must be contiguous CUDA float32 [P, 3]")
        _check_disjoint([means3D, xyz["first"], xyz["second"], dc, rest, dc_first,
                         dc_second, rest_first, rest_second],
                        "positions, their moments and the SH buffers must be disjoint")
        state["xyz"] = dict(first=xyz["first"], second=xyz["second"],
                            rate=float(xyz["rate"]), bias1=float(xyz["bias1"]),
                            bias2_sqrt=float(xyz["bias2_sqrt"]))
    return state


def rasterize_gaussians_backward_consume(bg, means3D, radii, colors, opacities, scales,
                                         rotations, scale_modifier, cov3D_precomp, viewmatrix,
                                         projmatrix, tanfovx, tanfovy, dL_dout_color,
                                         dL_dout_invdepth, sh, degree, campos, geomBuffer, R,
                                         binningBuffer, imageBuffer, antialiasing, debug, dc,
                                         rest, dc_first, dc_second, rest_first, rest_second,
                                         bias1, bias2_sqrt, *, xyz=None):
    _check(sh.dim() == 3 and sh.shape[1] == MAX_SH_COEFFS, "unsupported SH layout")
    consume = _consume_state(means3D, degree, dc, rest, dc_first, dc_second, rest_first,
                             rest_second, bias1, bias2_sqrt, xyz)
    return _backward(bg, means3D, radii, colors, opacities, scales, rotations, scale_modifier,
                     cov3D_precomp, viewmatrix, projmatrix, tanfovx, tanfovy, dL_dout_color,
                     dL_dout_invdepth, sh.contiguous(), None, None, degree, campos, geomBuffer,
                     R, binningBuffer, imageBuffer, antialiasing, consume)


def rasterize_gaussians_backward_consume_direct(bg, means3D, radii, colors, opacities, scales,
                                                rotations, scale_modifier, cov3D_precomp,
                                                viewmatrix, projmatrix, tanfovx, tanfovy,
                                                dL_dout_color, dL_dout_invdepth, sh, degree,
                                                campos, geomBuffer, R, binningBuffer,
                                                imageBuffer, antialiasing, debug, dc, rest,
                                                dc_first, dc_second, rest_first, rest_second,
                                                bias1, bias2_sqrt, *, xyz=None):
    _check_direct(means3D, dc, rest, degree)
    _check(sh.numel() == 0, "direct input path needs no coefficient snapshot")
    _check_disjoint([dc, rest, dc_first, dc_second, rest_first, rest_second],
                    "direct SH coefficient and moment buffers must be disjoint")
    consume = _consume_state(means3D, degree, dc, rest, dc_first, dc_second, rest_first,
                             rest_second, bias1, bias2_sqrt, xyz)
    return _backward(bg, means3D, radii, colors, opacities, scales, rotations, scale_modifier,
                     cov3D_precomp, viewmatrix, projmatrix, tanfovx, tanfovy, dL_dout_color,
                     dL_dout_invdepth, None, dc, rest, degree, campos, geomBuffer, R,
                     binningBuffer, imageBuffer, antialiasing, consume)


def mark_visible(means3D, viewmatrix, projmatrix):
    """Gaussians in front of the near plane (camera z > 0.2)."""
    p = means3D.contiguous()
    v = viewmatrix.contiguous().reshape(16)
    z = p[:, 0] * v[2] + p[:, 1] * v[6] + p[:, 2] * v[10] + v[14]
    return z > 0.2


# ----------------------------------------------------------------------------
# Autograd front end (the trainer's GaussianRasterizer).

class GaussianRasterizationSettings(NamedTuple):
    image_height: int
    image_width: int
    tanfovx: float
    tanfovy: float
    bg: torch.Tensor
    scale_modifier: float
    viewmatrix: torch.Tensor
    projmatrix: torch.Tensor
    sh_degree: int
    campos: torch.Tensor
    prefiltered: bool
    debug: bool
    antialiasing: bool = False


class _RasterizeGaussians(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means3D, means2D, sh, colors_precomp, opacities, scales, rotations,
                cov3Ds_precomp, settings):
        s = settings
        num, color, radii, geom, binning, image, invdepth = rasterize_gaussians(
            s.bg, means3D, colors_precomp, opacities, scales, rotations, s.scale_modifier,
            cov3Ds_precomp, s.viewmatrix, s.projmatrix, s.tanfovx, s.tanfovy, s.image_height,
            s.image_width, sh, s.sh_degree, s.campos, s.prefiltered, s.antialiasing, s.debug)
        ctx.settings, ctx.num = settings, num
        ctx.save_for_backward(colors_precomp, means3D, scales, rotations, cov3Ds_precomp,
                              radii, sh, opacities, geom, binning, image)
        return color, radii, invdepth

    @staticmethod
    def backward(ctx, grad_color, _grad_radii, grad_invdepth):
        s = ctx.settings
        (colors, means3D, scales, rotations, cov3D, radii, sh, opacities, geom, binning,
         image) = ctx.saved_tensors
        g2d, gcol, gop, gmean, gcov, gsh, gscale, grot = rasterize_gaussians_backward(
            s.bg, means3D, radii, colors, opacities, scales, rotations, s.scale_modifier,
            cov3D, s.viewmatrix, s.projmatrix, s.tanfovx, s.tanfovy, grad_color,
            grad_invdepth, sh, s.sh_degree, s.campos, geom, ctx.num, binning, image,
            s.antialiasing, s.debug)
        return (gmean, g2d, gsh if sh.numel() else None, gcol if colors.numel() else None,
                gop, gscale if scales.numel() else None, grot if rotations.numel() else None,
                gcov if cov3D.numel() else None, None)


class GaussianRasterizer(torch.nn.Module):
    def __init__(self, raster_settings):
        super().__init__()
        self.raster_settings = raster_settings

    def markVisible(self, positions):
        with torch.no_grad():
            s = self.raster_settings
            return mark_visible(positions, s.viewmatrix, s.projmatrix)

    def forward(self, means3D, means2D, opacities, shs=None, colors_precomp=None, scales=None,
                rotations=None, cov3D_precomp=None):
        if (shs is None) == (colors_precomp is None):
            raise Exception("Please provide excatly one of either SHs or precomputed colors!")
        if ((scales is None or rotations is None) and cov3D_precomp is None) or (
                (scales is not None or rotations is not None) and cov3D_precomp is not None):
            raise Exception("Please provide exactly one of either scale/rotation pair or "
                            "precomputed 3D covariance!")
        empty = torch.empty(0, device=means3D.device)
        return _RasterizeGaussians.apply(
            means3D, means2D, empty if shs is None else shs,
            empty if colors_precomp is None else colors_precomp, opacities,
            empty if scales is None else scales, empty if rotations is None else rotations,
            empty if cov3D_precomp is None else cov3D_precomp, self.raster_settings)


# ----------------------------------------------------------------------------
# Pixel stage on already projected 2D Gaussians (benchmark and tests).

def forward_2d(mean2d, conic_opacity, rgb, depth, radii, width, height, bg):
    """Bins, sorts and composites projected Gaussians (mean2d [P,2] px,
    conic_opacity [P,4], rgb [P,3], depth [P], radii [P] int32). Returns
    (num_rendered, color [3,H,W], state) with state for render_backward_2d."""
    device = mean2d.device
    P = mean2d.shape[0]
    color = torch.empty((3, height, width), dtype=torch.float32, device=device)
    invdepth = torch.empty((1, height, width), dtype=torch.float32, device=device)
    buffers = _Buffers(device)
    num = ctypes.c_int(0)
    keep = [t.contiguous() for t in (mean2d, conic_opacity, rgb, depth, radii, bg)]
    native.check(native.library().clad3dgs_raster_forward_2d(
        P, *[t.data_ptr() for t in keep[:5]], int(width), int(height), keep[5].data_ptr(),
        ctypes.cast(buffers.callback, ctypes.c_void_p), None, color.data_ptr(),
        invdepth.data_ptr(), ctypes.byref(num), native.stream_handle()), "forward_2d")
    state = dict(P=P, width=int(width), height=int(height), bg=keep[5], geom=buffers.get(0),
                 binning=buffers.get(2), image=buffers.get(1), num_rendered=num.value)
    return num.value, color, invdepth, state


def count_accumulation_2d(state):
    """Atomic counts of the pixel backward on a forward_2d state (a counting
    pass, not the backward): dict(pairs, mode1_per_field, mode2_reductions);
    see clad3dgs_raster_count_accumulation."""
    counts = torch.zeros(3, dtype=torch.int64, device=state["geom"].device)
    native.check(native.library().clad3dgs_raster_count_accumulation(
        state["P"], state["width"], state["height"], state["geom"].data_ptr(),
        state["binning"].data_ptr(), state["num_rendered"], state["image"].data_ptr(),
        counts.data_ptr(), native.stream_handle()), "count_accumulation_2d")
    pairs, mode1, mode2 = (int(x) for x in counts.cpu().tolist())
    return dict(pairs=pairs, mode1_per_field=mode1, mode2_reductions=mode2)


def render_backward_2d(state, dpixels, grads, mode=None, dinvdepth_pixels=None):
    """Pixel backward into grads = dict(dmean2d [P,3], dconic [P,4],
    dopacity [P], dcolor [P,3], dinvdepth [P] or None), accumulated."""
    mode = pixel_accumulation if mode is None else mode
    native.check(native.library().clad3dgs_raster_render_backward(
        state["P"], state["width"], state["height"], state["bg"].data_ptr(),
        state["geom"].data_ptr(), state["binning"].data_ptr(), state["num_rendered"],
        state["image"].data_ptr(), dpixels.data_ptr(), native.ptr(dinvdepth_pixels),
        grads["dmean2d"].data_ptr(), grads["dconic"].data_ptr(), grads["dopacity"].data_ptr(),
        grads["dcolor"].data_ptr(), native.ptr(grads.get("dinvdepth")), int(mode),
        native.stream_handle()), "render_backward_2d")
