"""Data-parallel Gaussian training on one node: one camera view per GPU,
parameters replicated on every GPU, Adam moments sharded by Gaussian index.

The reference trains on one GPU; this module is the multi-GPU form of its
per-Gaussian update path. Per step on every rank:

1. `activate`: exp(log-scale), normalised quaternion, sigmoid(opacity logit),
   keeping |q| for the quaternion VJP (activation.py:24-37);
2. render the rank's view, L1 loss against its target, rasterizer backward
   into this rank's gradient arrays (gradients of the activated scaling,
   rotation and opacity);
3. the exchange + update of `ShardedAdam.step`:

   * ``exchange="peer"`` (default with more than one GPU): parameters and
     gradients live in CUDA-IPC memory that every rank maps. After a barrier,
     each rank's `clad3dgs_shard_update` kernel reads the gradients of the
     Gaussians it owns from every rank's memory (in rank order), applies the
     activation VJPs and torch-fused Adam with its own moments, and stores the
     new parameters into every rank's replica; a second barrier ends the step.
     One kernel does reduce-scatter, Adam and all-gather.
   * ``exchange="collective"``: reduce-scatter of each gradient group, the same
     kernel over the local share (one source, one replica), all-gather of each
     parameter group through torch.distributed (the NCCL baseline; gloo in the
     CPU tests).

   What a rank publishes for the SH coefficients (``sh_exchange``):

   * ``"seeds"`` (default on CUDA unless the exchange is the collective one
     with more than one rank): the rasterizer backward stops before the SH
     backward (consume_sh = 2) and the rank publishes its view's colour seeds
     (dL/dcolour with clamped channels zeroed, and a drawn flag: 16 B per
     Gaussian instead of 192 B of SH gradients) and its camera position; the
     owner of a share evaluates every view's SH backward and view-direction
     adjoint inside the update, summed in rank order, bit-identical to the
     gradient form.
   * ``"colours"`` (peer exchange or one rank): the seed form, and in
     addition no rank holds the other shares' SH coefficients. The owner of a
     share renders, inside the update, each rank's colours for that rank's
     next camera (declared with the step) and stores 12 B per Gaussian into
     the rank's colour array instead of 192 B of coefficients into its
     replica; the rank renders from those colours (colors_precomp). The owner
     keeps which channels its clamp cut and masks the seeds with them. Same
     parameters, bit for bit, as the seed form; before the first step
     `prime` renders the first colours.
   * ``"grads"``: each rank writes its full SH gradients and the update sums
     them (the form a collective reduce-scatter needs).

Barriers are one-element all-reduces on the compute stream, so they order the
GPUs' streams without a host wait.

Groups per Gaussian (59 floats): xyz 3, SH 48 ([16][3]; coefficient 0 uses the
f_dc rate, 1..15 f_rest), scaling 3, rotation 4, opacity 1. Each group is one
[N][k] array, so a rank's share of a group is one contiguous span.
"""

from __future__ import annotations

import ctypes
import math
from typing import NamedTuple

import torch
import torch.distributed as dist

import _native as native

GROUPS = (("xyz", 3), ("sh", 48), ("scaling", 3), ("rotation", 4), ("opacity", 1))
WIDTH = dict(GROUPS)
FLOATS_PER_GAUSSIAN = sum(k for _, k in GROUPS)  # 59
RATE_NAMES = ("xyz", "f_dc", "f_rest", "scaling", "rotation", "opacity")
# The 3DGS trainer's default learning rates (position rate before its schedule).
DEFAULT_RATES = dict(xyz=0.00016, f_dc=0.0025, f_rest=0.000125, scaling=0.005,
                     rotation=0.001, opacity=0.025)


def plan(n, world):
    """(padded Gaussian count, share per rank): equal shares, multiples of 4.
    Padding Gaussians are never rendered; their gradients stay zero, so Adam
    leaves them unchanged."""
    if n < 0 or world < 1:
        raise ValueError("plan: need n >= 0 and world >= 1")
    unit = 4 * world
    padded = -(-n // unit) * unit
    return padded, padded // world


def group_offsets(padded):
    """Float offset of each group in a 59 x padded slab."""
    offsets, at = {}, 0
    for name, k in GROUPS:
        offsets[name] = at
        at += k * padded
    return offsets


def carve(slab, rows):
    """Views [rows, k] of each group of a flat slab."""
    out = {}
    for name, off in group_offsets(rows).items():
        k = WIDTH[name]
        out[name] = slab[off:off + k * rows].view(rows, k)
    return out


class _DeviceArray:
    """A raw device allocation seen by torch through __cuda_array_interface__."""

    def __init__(self, address, count):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": "<f4",
                                         "data": (int(address), False), "version": 3,
                                         "strides": None}


class ShardStep(NamedTuple):
    """Arguments of one exchange + update call (tensors or raw addresses)."""
    begin: int
    end: int
    grad_origin: int
    grads: list       # [ranks][5]
    params: list      # [ranks][5]
    local: int
    first: list       # [5]
    second: list      # [5]
    saved_scaling: object
    saved_opacity: object
    saved_norm: object
    rates: tuple      # 6 rates: xyz, f_dc, f_rest, scaling, rotation, opacity
    bias1: float
    bias2_sqrt: float
    seeds: list = None    # seed form: [ranks] colour seed arrays [N][4]
    cameras: list = None  # seed form: [ranks] camera positions (3 floats)
    degree: int = 3       # seed form: SH degree
    colours: list = None       # colour form: [ranks] colour arrays [N][3]
    next_cameras: list = None  # colour form: [ranks] next camera positions
    clamp_bits: object = None  # colour form: the share's clamp bits [end - begin]


def _address(x):
    if x is None:
        return None
    return int(x) if isinstance(x, int) else x.data_ptr()


def _arguments(s: ShardStep):
    args = native.ShardUpdateArgs()
    args.begin, args.end, args.grad_origin = s.begin, s.end, s.grad_origin
    args.ranks, args.local = len(s.grads), s.local
    for q in range(len(s.grads)):
        for g in range(len(GROUPS)):
            args.grads[q][g] = _address(s.grads[q][g])
            args.params[q][g] = _address(s.params[q][g])
    for g in range(len(GROUPS)):
        args.first[g] = _address(s.first[g])
        args.second[g] = _address(s.second[g])
    args.saved_scaling = _address(s.saved_scaling)
    args.saved_opacity = _address(s.saved_opacity)
    args.saved_norm = _address(s.saved_norm)
    for r, rate in enumerate(s.rates):
        args.rates[r] = float(rate)
    args.bias1, args.bias2_sqrt = float(s.bias1), float(s.bias2_sqrt)
    if s.seeds is not None:
        for q in range(len(s.seeds)):
            args.seeds[q] = _address(s.seeds[q])
            args.cameras[q] = _address(s.cameras[q])
    args.degree = int(s.degree)
    if s.colours is not None:
        for q in range(len(s.colours)):
            args.colours[q] = _address(s.colours[q])
            args.next_cameras[q] = _address(s.next_cameras[q])
        args.clamp_bits = _address(s.clamp_bits)
    return args


def native_update(s: ShardStep, stream=None):
    """clad3dgs_shard_update on the current stream."""
    native.check(native.library().clad3dgs_shard_update(ctypes.byref(_arguments(s)),
                                                        native.stream_handle(stream)),
                 "shard update")


def native_colours(s: ShardStep, stream=None):
    """clad3dgs_shard_colours (the colour form's first colours) on the current
    stream."""
    native.check(native.library().clad3dgs_shard_colours(ctypes.byref(_arguments(s)),
                                                         native.stream_handle(stream)),
                 "shard colours")


class ShardedAdam:
    """Replicated parameters, per-view gradients and sharded Adam state of n
    Gaussians across the ranks of `group` (or one process without one).

    Attributes: `params` / `grads` (dicts of [padded, k] views, replicated /
    this rank's view), `first` / `second` (moments of the share [begin, end)),
    `saved` (activated scaling / rotation / opacity and |q|, [padded, .]); in
    seed form `seeds` ([padded, 4], this rank's view) and `camera` (its
    position, 3 floats), written before each step; in colour form also
    `next_camera` (the position this rank renders from at the next step,
    written before each step) and `colours` ([padded, 3], what the owners
    rendered for it; the replica's SH coefficients are current only in this
    rank's share: `gather_sh` brings the others in).
    """

    def __init__(self, n, rates=None, *, group=None, exchange=None, device=None,
                 update=None, sh_exchange=None, degree=3, gate=None):
        self.group = group
        # rank_health.StepGate: when given, every step first settles on the
        # host that all ranks are present (before any collective is enqueued).
        self.gate = gate
        self.distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if self.distributed else 1
        self.rank = dist.get_rank(group) if self.distributed else 0
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        if exchange is None:
            exchange = "peer" if self.world > 1 and self.device.type == "cuda" else "collective"
        if exchange not in ("peer", "collective"):
            raise ValueError("exchange must be 'peer' or 'collective'")
        if exchange == "peer" and self.device.type != "cuda":
            raise ValueError("the peer exchange needs CUDA devices")
        self.exchange = exchange
        if sh_exchange is None:
            collective = exchange == "collective" and self.world > 1
            sh_exchange = "seeds" if self.device.type == "cuda" and not collective else "grads"
        if sh_exchange not in ("seeds", "colours", "grads"):
            raise ValueError("sh_exchange must be 'seeds', 'colours' or 'grads'")
        if sh_exchange != "grads" and exchange == "collective" and self.world > 1:
            raise ValueError("the collective exchange reduces SH gradients: use 'grads'")
        if sh_exchange != "grads" and self.device.type != "cuda":
            raise ValueError(f"the {sh_exchange[:-1]} form needs CUDA devices")
        self.sh_exchange = sh_exchange
        self.degree = int(degree)
        self.rates = dict(DEFAULT_RATES if rates is None else rates)
        missing = [r for r in RATE_NAMES if r not in self.rates]
        if missing:
            raise ValueError(f"missing learning rates: {missing}")
        self.n = int(n)
        self.padded, self.share = plan(self.n, self.world)
        self.begin = self.rank * self.share
        self.end = self.begin + self.share
        self.t = 0
        self._settled = 0  # gate passes outside the steps
        self._update = update or native_update
        total = FLOATS_PER_GAUSSIAN * self.padded
        self._own = []
        self._peers = []
        # Seed slab: the camera position and the next one (4 floats each, so
        # the seeds stay 16-byte aligned), then [padded, 4] seeds; padding
        # Gaussians keep zero seeds. Colour form: [padded, 3] colours after them.
        seeded = sh_exchange != "grads"
        coloured = sh_exchange == "colours"
        seed_total = (8 + 4 * self.padded + (3 * self.padded if coloured else 0)
                      if seeded else 0)
        if exchange == "peer" and self.world > 1:
            param_slab, param_handle = self._ipc_slab(total)
            grad_slab, grad_handle = self._ipc_slab(total)
            seed_slab, seed_handle = (self._ipc_slab(seed_total) if seed_total
                                      else (None, None))
        else:
            param_slab = torch.zeros(total, dtype=torch.float32, device=self.device)
            grad_slab = torch.zeros(total, dtype=torch.float32, device=self.device)
            seed_slab = (torch.zeros(seed_total, dtype=torch.float32, device=self.device)
                         if seed_total else None)
            seed_handle = None
        self.param_slab, self.grad_slab, self.seed_slab = param_slab, grad_slab, seed_slab
        self.params = carve(param_slab, self.padded)
        self.grads = carve(grad_slab, self.padded)
        self.colours = self.next_camera = self.clamp_bits = None
        if seed_slab is not None:
            if exchange == "peer" and self.world > 1:
                seed_slab.zero_()
            self.camera = seed_slab[:3]
            self.next_camera = seed_slab[4:7]
            self.seeds = seed_slab[8:8 + 4 * self.padded].view(self.padded, 4)
            if coloured:
                self.colours = seed_slab[8 + 4 * self.padded:].view(self.padded, 3)
                self.clamp_bits = torch.zeros(self.share, dtype=torch.int32,
                                              device=self.device)
        else:
            self.camera = self.seeds = None
        zeros = lambda *s: torch.zeros(s, dtype=torch.float32, device=self.device)
        self.first = carve(zeros(FLOATS_PER_GAUSSIAN * self.share), self.share)
        self.second = carve(zeros(FLOATS_PER_GAUSSIAN * self.share), self.share)
        self.saved = dict(scaling=zeros(self.padded, 3), rotation=zeros(self.padded, 4),
                          opacity=zeros(self.padded, 1), norm=zeros(self.padded))
        if exchange == "collective" and self.world > 1:
            self.reduced = carve(zeros(FLOATS_PER_GAUSSIAN * self.share), self.share)
        self._flag = zeros(1)
        if exchange == "peer" and self.world > 1:
            self._open_peers(param_handle, grad_handle, seed_handle)

    # -- CUDA IPC memory -------------------------------------------------
    def _ipc_slab(self, count):
        address = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * native.IPC_HANDLE_BYTES)()
        native.check(native.library().clad3dgs_ipc_alloc(count * 4, ctypes.byref(address),
                                                         handle), "ipc alloc")
        self._own.append(address.value)
        tensor = torch.as_tensor(_DeviceArray(address.value, count), device=self.device)
        return tensor, bytes(handle)

    def _open_peers(self, param_handle, grad_handle, seed_handle=None):
        handles = [param_handle, grad_handle] + ([seed_handle] if seed_handle else [])
        mine = torch.tensor(list(b"".join(handles)), dtype=torch.uint8, device=self.device)
        every = torch.empty(self.world * mine.numel(), dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(every, mine, group=self.group)
        every = every.view(self.world, len(handles), native.IPC_HANDLE_BYTES).cpu()
        offsets = group_offsets(self.padded)
        self.peer_params, self.peer_grads = [], []
        self.peer_seeds, self.peer_cameras = [], []
        self.peer_next_cameras, self.peer_colours = [], []
        for q in range(self.world):
            if q == self.rank:
                bases = [self.param_slab.data_ptr(), self.grad_slab.data_ptr()]
                if seed_handle:
                    bases.append(self.seed_slab.data_ptr())
            else:
                bases = []
                for which in range(len(handles)):
                    handle = (ctypes.c_ubyte * native.IPC_HANDLE_BYTES)(
                        *every[q, which].tolist())
                    address = ctypes.c_void_p()
                    native.check(native.library().clad3dgs_ipc_open(handle,
                                                                     ctypes.byref(address)),
                                 "ipc open")
                    self._peers.append(address.value)
                    bases.append(address.value)
            self.peer_params.append([bases[0] + 4 * offsets[name] for name, _ in GROUPS])
            self.peer_grads.append([bases[1] + 4 * offsets[name] for name, _ in GROUPS])
            if seed_handle:
                self.peer_cameras.append(bases[2])
                self.peer_next_cameras.append(bases[2] + 16)
                self.peer_seeds.append(bases[2] + 32)
                self.peer_colours.append(bases[2] + 32 + 16 * self.padded)

    def close(self):
        """Unmaps the peers' memory and frees this rank's (collective call)."""
        if not self._own and not self._peers:
            return
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        if self.distributed and self.world > 1:
            dist.barrier(group=self.group)
        for address in self._peers:
            native.check(native.library().clad3dgs_ipc_close(address), "ipc close")
        self._peers = []
        if self.distributed and self.world > 1:
            dist.barrier(group=self.group)
        self.params = self.grads = self.seeds = self.camera = None
        self.colours = self.next_camera = None
        self.param_slab = self.grad_slab = self.seed_slab = None
        for address in self._own:
            native.check(native.library().clad3dgs_ipc_free(address), "ipc free")
        self._own = []

    def leave(self):
        """This rank takes part in no further step: the other ranks' next gate
        raises RankFailure instead of waiting in a collective."""
        if self.gate is not None:
            self.gate.leave()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- per step --------------------------------------------------------
    def load(self, values):
        """Copies initial parameter values (dict of [n, k]) into the replica."""
        for name, k in GROUPS:
            v = values[name].reshape(self.n, k)
            self.params[name][:self.n].copy_(v)

    def state_dict(self):
        """This rank's part of a checkpoint (collective in colour form, whose
        replicas are first completed by `gather_sh`): the step counter, the
        parameters of the n Gaussians and the moments of this rank's share."""
        self.gather_sh()
        return {"t": self.t, "n": self.n, "world": self.world, "rank": self.rank,
                "params": {k: v[:self.n].detach().cpu().clone() for k, v in self.params.items()},
                "first": {k: v.detach().cpu().clone() for k, v in self.first.items()},
                "second": {k: v.detach().cpu().clone() for k, v in self.second.items()}}

    def load_state_dict(self, state):
        """Restores `state_dict` output of the same rank of a group of the
        same size (the moments are sharded by Gaussian index). In colour form
        the colours must be made again (`prime`) before the next step."""
        if (state["n"], state["world"], state["rank"]) != (self.n, self.world, self.rank):
            raise ValueError(
                f"checkpoint of rank {state['rank']} of {state['world']} over {state['n']} "
                f"Gaussians does not fit rank {self.rank} of {self.world} over {self.n}")
        self.load(state["params"])
        for name, _ in GROUPS:
            self.first[name].copy_(state["first"][name])
            self.second[name].copy_(state["second"][name])
        self.t = int(state["t"])

    def activate(self):
        """Activated scaling / rotation / opacity and |q| for every Gaussian."""
        p, s = self.params, self.saved
        native.check(native.library().clad3dgs_activate(
            self.padded, p["scaling"].data_ptr(), p["rotation"].data_ptr(),
            p["opacity"].data_ptr(), s["scaling"].data_ptr(), s["rotation"].data_ptr(),
            s["opacity"].data_ptr(), s["norm"].data_ptr(), native.stream_handle()),
            "activate")
        return s

    def zero_grad(self):
        self.grad_slab.zero_()

    def zero_accumulated(self):
        """Zeroes only the gradient arrays the rasterizer backward accumulates
        into (positions, opacity); it writes the others outright."""
        self.grads["xyz"].zero_()
        self.grads["opacity"].zero_()

    def _barrier(self):
        dist.all_reduce(self._flag, group=self.group)

    def _settle(self, what):
        """The step gate for a collective outside the step (priming the
        colours, gathering the SH): every rank present, or RankFailure."""
        if self.gate is not None and self.world > 1:
            self._settled += 1
            self.gate.arrive_and_wait(f"{what}-{self._settled}")

    def _shard_step(self, grads, params, grad_origin, local, seeds=None, cameras=None,
                    colours=None, next_cameras=None):
        t = max(self.t, 1)  # `prime` comes before the first step and reads no rate
        return ShardStep(
            begin=self.begin, end=self.end, grad_origin=grad_origin, grads=grads,
            params=params, local=local, first=[self.first[n] for n, _ in GROUPS],
            second=[self.second[n] for n, _ in GROUPS], saved_scaling=self.saved["scaling"],
            saved_opacity=self.saved["opacity"], saved_norm=self.saved["norm"],
            rates=tuple(self.rates[r] for r in RATE_NAMES), bias1=1.0 - 0.9 ** t,
            bias2_sqrt=math.sqrt(1.0 - 0.999 ** t), seeds=seeds, cameras=cameras,
            degree=self.degree, colours=colours, next_cameras=next_cameras,
            clamp_bits=self.clamp_bits if colours is not None else None)

    def _peer_step(self):
        """The step's arguments over every rank's memory (one rank: its own)."""
        names = [n for n, _ in GROUPS]
        seeded = self.sh_exchange != "grads"
        coloured = self.sh_exchange == "colours"
        if self.world == 1:
            return self._shard_step([[self.grads[n] for n in names]],
                                    [[self.params[n] for n in names]], 0, 0,
                                    [self.seeds] if seeded else None,
                                    [self.camera] if seeded else None,
                                    [self.colours] if coloured else None,
                                    [self.next_camera] if coloured else None)
        return self._shard_step(self.peer_grads, self.peer_params, 0, self.rank,
                                self.peer_seeds if seeded else None,
                                self.peer_cameras if seeded else None,
                                self.peer_colours if coloured else None,
                                self.peer_next_cameras if coloured else None)

    def prime(self):
        """Colour form, before the first step (collective): every owner renders
        its share's colours for every rank's `next_camera` from the current
        parameters."""
        if self.sh_exchange != "colours":
            raise ValueError("prime belongs to the colour form")
        self._settle("colours")
        if self.world > 1:
            self._barrier()
        native_colours(self._peer_step())
        if self.world > 1:
            self._barrier()

    def gather_sh(self):
        """Colour form: brings the other shares' SH coefficients into this
        rank's replica (collective; the seed and gradient forms keep every
        replica current, so there it does nothing)."""
        if self.sh_exchange != "colours" or self.world == 1:
            return self.params["sh"]
        self._settle("gather")
        full = self.params["sh"].view(-1)
        mine = full[48 * self.begin:48 * self.end].clone()
        dist.all_gather_into_tensor(full, mine, group=self.group)
        return self.params["sh"]

    def step(self):
        """Sums the ranks' gradients of this rank's share, runs Adam on it and
        brings every replica up to date."""
        self.t += 1
        if self.gate is not None and self.world > 1:
            self.gate.arrive_and_wait(self.t)
        names = [n for n, _ in GROUPS]
        if self.world == 1:
            self._update(self._peer_step())
        elif self.exchange == "peer":
            self._barrier()
            self._update(self._peer_step())
            self._barrier()
        else:
            for n in names:
                dist.reduce_scatter_tensor(self.reduced[n].view(-1), self.grads[n].view(-1),
                                           group=self.group)
            self._update(self._shard_step([[self.reduced[n] for n in names]],
                                          [[self.params[n] for n in names]], self.begin, 0))
            for n in names:
                full = self.params[n].view(-1)
                k = WIDTH[n]
                dist.all_gather_into_tensor(full, full[self.begin * k:self.end * k],
                                            group=self.group)


# ---------------------------------------------------------------------------
# Cameras and the training step.

class Camera(NamedTuple):
    width: int
    height: int
    tan_x: float
    tan_y: float
    view: torch.Tensor      # [4, 4] column-major world-to-camera (renderer convention)
    proj: torch.Tensor      # [4, 4] column-major full projection
    campos: torch.Tensor    # [3]


def orbit_camera(index, count, *, radius=4.0, width=1920, height=1080,
                 fov_x=math.radians(60.0), device=None, znear=0.01, zfar=100.0):
    """Camera `index` of `count` on a horizontal circle of `radius` around the
    origin, looking at it (x right, y down, z forward)."""
    theta = 2.0 * math.pi * index / count
    pos = torch.tensor([radius * math.sin(theta), 0.0, -radius * math.cos(theta)],
                       dtype=torch.float64)
    forward = -pos / pos.norm()
    down0 = torch.tensor([0.0, 1.0, 0.0], dtype=torch.float64)
    right = torch.linalg.cross(down0, forward)
    right = right / right.norm()
    down = torch.linalg.cross(forward, right)
    w2c = torch.eye(4, dtype=torch.float64)
    w2c[0, :3], w2c[1, :3], w2c[2, :3] = right, down, forward
    w2c[:3, 3] = -(w2c[:3, :3] @ pos)
    tan_x = math.tan(fov_x / 2)
    tan_y = tan_x * height / width
    P = torch.zeros(4, 4, dtype=torch.float64)
    P[0, 0] = 1.0 / tan_x
    P[1, 1] = 1.0 / tan_y
    P[3, 2] = 1.0
    P[2, 2] = zfar / (zfar - znear)
    P[2, 3] = -(zfar * znear) / (zfar - znear)
    f32 = lambda t: t.to(torch.float32).contiguous().to(device)
    return Camera(width, height, tan_x, tan_y, f32(w2c.T), f32((P @ w2c).T), f32(pos))


class _Scratch:
    """Rasterizer scratch reused across steps (grown on demand)."""

    def __init__(self, device):
        self.device = device
        self.tensors = {}

        def allocate(_ctx, which, nbytes):
            t = self.tensors.get(int(which))
            if t is None or t.numel() < nbytes:
                t = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=self.device)
                self.tensors[int(which)] = t
            return t.data_ptr()

        self.callback = native.ALLOC_FN(allocate)


class DataParallelTrainer:
    """One training step per call: this rank renders its camera, takes the L1
    loss against its target, back-propagates into its gradient arrays, and the
    ranks exchange and update (ShardedAdam.step)."""

    def __init__(self, values, rates=None, *, degree=3, bg=(0.0, 0.0, 0.0), group=None,
                 exchange=None, device=None, pixel_accumulation=2, sh_exchange=None,
                 gate=None):
        n = int(values["xyz"].shape[0])
        self.adam = ShardedAdam(n, rates, group=group, exchange=exchange, device=device,
                                sh_exchange=sh_exchange, degree=degree, gate=gate)
        self.adam.load(values)
        self.n, self.degree = n, int(degree)
        self.mode = int(pixel_accumulation)
        dev = self.adam.device
        self.bg = torch.tensor(bg, dtype=torch.float32, device=dev)
        z = lambda *s: torch.zeros(s, dtype=torch.float32, device=dev)
        # The pixel backward's per-Gaussian targets (accumulated, so zeroed every
        # step) are carved from one buffer: one fill clears them all.
        self._accumulated = z(10 * n)
        acc = self._accumulated
        self.scratch_grads = dict(mean2d=acc[:3 * n].view(n, 3), colors=acc[3 * n:6 * n].view(n, 3),
                                  conic=acc[6 * n:].view(n, 4), cov=z(n, 6))
        self.radii = torch.zeros(n, dtype=torch.int32, device=dev)
        self.loss = z(1)
        self.buffers = _Scratch(dev)
        self.image = self.dimage = None
        self._declared = None  # colour form: the camera the colours were made for

    def close(self):
        self.adam.close()

    def state_dict(self):
        """This rank's checkpoint (collective in colour form)."""
        return self.adam.state_dict()

    def load_state_dict(self, state):
        """Restores `state_dict`; in colour form the next step primes the
        colours again from the camera it renders."""
        self.adam.load_state_dict(state)
        self._declared = None

    def prime(self, camera: Camera):
        """Colour form (collective): declares the camera of the first step and
        has the owners render its colours."""
        a = self.adam
        a.next_camera.copy_(camera.campos)
        a.prime()
        self._declared = camera

    def step(self, camera: Camera, target, next_camera: Camera = None):
        """Render, loss, backward and the exchange + update; returns the loss
        (a device tensor) and the number of tile instances rendered.

        Colour form: `next_camera` is the camera this rank renders at its
        next step (the update renders its colours), and `camera` must be the
        one declared so by the previous step (or the first camera, which
        primes the colours)."""
        a = self.adam
        if a.sh_exchange == "colours":
            if next_camera is None:
                raise ValueError("the colour form needs the next step's camera")
            if self._declared is None:
                self.prime(camera)
            elif camera is not self._declared:
                raise ValueError("the colour form renders the camera declared as "
                                 "next_camera at the previous step")
        loss, rendered = self.backward(camera, target)
        if a.sh_exchange == "colours":
            a.next_camera.copy_(next_camera.campos)
        a.step()
        if a.sh_exchange == "colours":
            self._declared = next_camera
        return loss, rendered

    def backward(self, camera: Camera, target):
        """Everything of a step before the exchange: this rank's gradients."""
        lib, a = native.library(), self.adam
        stream = native.stream_handle()
        n, H, W = self.n, camera.height, camera.width
        if self.image is None or self.image.shape != (3, H, W):
            self.image = torch.empty(3, H, W, dtype=torch.float32, device=a.device)
            self.dimage = torch.empty_like(self.image)
            self.invdepth = torch.empty(1, H, W, dtype=torch.float32, device=a.device)
        # Only atomically accumulated arrays need clearing: the positions'
        # and opacity gradients and the pixel backward's per-Gaussian targets
        # (the SH, scale, rotation and covariance adjoints and the seeds are
        # written outright).
        a.zero_accumulated()
        self._accumulated.zero_()
        self.loss.zero_()
        act = a.activate()
        p = a.params
        # Colour form: the owners' colours for this view stand for the SH.
        colours = a.colours.data_ptr() if a.sh_exchange == "colours" else None
        sh = None if colours else p["sh"].data_ptr()
        rendered = ctypes.c_int(0)
        native.check(lib.clad3dgs_raster_forward(
            n, self.degree, self.bg.data_ptr(), p["xyz"].data_ptr(), colours,
            act["opacity"].data_ptr(), act["scaling"].data_ptr(), 1.0,
            act["rotation"].data_ptr(), None, camera.view.data_ptr(), camera.proj.data_ptr(),
            camera.tan_x, camera.tan_y, H, W, sh, None, None,
            camera.campos.data_ptr(), 0, ctypes.cast(self.buffers.callback, ctypes.c_void_p),
            None, self.image.data_ptr(), self.invdepth.data_ptr(), self.radii.data_ptr(),
            ctypes.byref(rendered), stream), "rasterize (forward)")
        native.check(lib.clad3dgs_l1_loss(3 * H * W, self.image.data_ptr(), target.data_ptr(),
                                          self.dimage.data_ptr(), self.loss.data_ptr(),
                                          stream), "l1 loss")
        g, s = a.grads, self.scratch_grads
        seeded = a.sh_exchange != "grads"
        geom = self.buffers.tensors.get(0)
        image = self.buffers.tensors.get(1)
        binning = self.buffers.tensors.get(2)
        native.check(lib.clad3dgs_raster_backward(
            n, self.degree, self.bg.data_ptr(), p["xyz"].data_ptr(), self.radii.data_ptr(),
            colours, act["opacity"].data_ptr(), act["scaling"].data_ptr(), 1.0,
            act["rotation"].data_ptr(), None, camera.view.data_ptr(), camera.proj.data_ptr(),
            camera.tan_x, camera.tan_y, H, W, self.dimage.data_ptr(),
            None, sh, None, None,
            camera.campos.data_ptr(), geom.data_ptr(), rendered.value,
            binning.data_ptr() if binning is not None else None, image.data_ptr(), 0,
            s["mean2d"].data_ptr(), s["colors"].data_ptr(), g["opacity"].data_ptr(),
            g["xyz"].data_ptr(), s["cov"].data_ptr(), g["sh"].data_ptr(),
            g["scaling"].data_ptr(), g["rotation"].data_ptr(), s["conic"].data_ptr(),
            None, self.mode, 2 if seeded else 0, None, None, None, None, None, None,
            native.TorchAdamConfig(1.0, 1.0), None, None, 0.0, native.TorchAdamConfig(1.0, 1.0),
            stream), "rasterize (backward)")
        if seeded:
            # This view's colour seeds and camera for the SH backward in the update.
            native.check(lib.clad3dgs_raster_sh_seeds(
                n, self.radii.data_ptr(), geom.data_ptr(), s["colors"].data_ptr(),
                a.seeds.data_ptr(), stream), "SH seeds")
            a.camera.copy_(camera.campos)
        return self.loss, rendered.value
