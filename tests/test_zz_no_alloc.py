"""The allocation-free host-buffer step, for callers that cannot call cudaMalloc.

Some callers embed this library in a host application that owns all device
memory through its own allocator or a fixed budget, or call it from a hot loop
that must not pay for an allocation's implicit synchronisation; for them
clad3dgs_gaussian_step_host_static stages chunks in a fixed device array
inside the library instead of a workspace the caller allocates. These checks
call it through the C ABI and compare it with the workspace-based
clad3dgs_gaussian_step_host, bit for bit (the tolerance every fused-step test
here uses), on two calls in a row, and check that a chunk too large for the
fixed array is refused without touching the caller's buffers. The file is named
to run last and needs nothing from the other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu


def _host_state(n, seed):
    sh = cases.sh_problem(n, seed=seed, moments=True)
    act = cases.activation_problem(n, seed=seed + 1, moments=True)
    h = {k: torch.from_numpy(np.ascontiguousarray(v)).pin_memory() for k, v in sh.items()}
    ha = {k: [torch.from_numpy(np.ascontiguousarray(x)).pin_memory() for x in act[k]]
          for k in ("params", "seeds", "saved", "first", "second")}
    return h, ha, act["rates"]


def _arguments(h, ha, rates, step):
    import _native as native

    b1, b2 = cases.bias(step)
    arrays = [native.pointer_array([t.data_ptr() for t in ha[k]])
              for k in ("params", "seeds", "saved", "first", "second")]
    head = [h[k].data_ptr() for k in ("means", "radii", "clamped", "camera", "seed", "dm",
                                       "dc", "rest", "dc_first", "dc_second", "rest_first",
                                       "rest_second")]
    return (head, native.TorchAdamConfig(b1, b2),
            [ctypes.cast(a, ctypes.POINTER(ctypes.c_void_p)) for a in arrays],
            native.doubles(rates), native.floats([b1] * 3), native.floats([b2] * 3))


def _snapshot(h, ha):
    out = [v.numpy().copy() for k, v in sorted(h.items())]
    out += [x.numpy().copy() for k in sorted(ha) for x in ha[k]]
    return out


def _identical(a, b):
    return all(((x.view(np.uint8) == y.view(np.uint8)).all()) for x, y in zip(a, b))


@pytest.mark.parametrize("n,chunk", [(100_003, 0), (5000, 1024)])
def test_static_step_matches_workspace_step_on_two_calls(cuda, n, chunk):
    import consume
    import _native as native

    lib = native.library()
    static_state = _host_state(n, seed=21)
    workspace_state = _host_state(n, seed=21)
    ws_chunk = 8192
    workspace = torch.empty(consume.host_step_workspace(ws_chunk), dtype=torch.uint8,
                            device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    for step in (1, 2):
        head, cfg, arrays, rates, b1, b2 = _arguments(*static_state, step)
        status = lib.clad3dgs_gaussian_step_host_static(n, 3, *head, cfg, *arrays, rates,
                                                        b1, b2, chunk, stream)
        assert status == native.OK, lib.clad3dgs_last_error()
        head, cfg, arrays, rates, b1, b2 = _arguments(*workspace_state, step)
        status = lib.clad3dgs_gaussian_step_host(n, 3, *head, cfg, *arrays, rates, b1, b2,
                                                 workspace.data_ptr(), workspace.numel(),
                                                 ws_chunk, stream)
        assert status == native.OK, lib.clad3dgs_last_error()
        assert _identical(_snapshot(*static_state[:2]), _snapshot(*workspace_state[:2])), step
    assert native.fault_status() == 0


def test_static_step_rejects_chunks_beyond_the_fixed_array(cuda):
    import _native as native

    lib = native.library()
    n = 1000
    state = _host_state(n, seed=5)
    before = _snapshot(*state[:2])
    head, cfg, arrays, rates, b1, b2 = _arguments(*state, 1)
    for chunk in (1 << 22, 100):  # far too large for 48 MiB; not a multiple of 64
        status = lib.clad3dgs_gaussian_step_host_static(n, 3, *head, cfg, *arrays, rates,
                                                        b1, b2, chunk, 0)
        assert status == native.INVALID_ARGUMENT
        assert b"staging" in lib.clad3dgs_last_error()
    assert _identical(_snapshot(*state[:2]), before)


def _static_limit(lib, native, state):
    """The largest chunk the fixed array takes, as the rejection message states."""
    import re

    head, cfg, arrays, rates, b1, b2 = _arguments(*state, 1)
    status = lib.clad3dgs_gaussian_step_host_static(1000, 3, *head, cfg, *arrays, rates,
                                                    b1, b2, 1 << 22, 0)
    assert status == native.INVALID_ARGUMENT
    return int(re.search(rb"up to (\d+)", lib.clad3dgs_last_error()).group(1))


def test_static_step_at_its_chunk_limit(cuda):
    """A chunk exactly at the limit runs and matches the workspace step bit for
    bit; one step of 64 above it is refused before anything is written. The
    limit uses the array's 48 MiB: about 65K Gaussians at 767 staged bytes each."""
    import consume
    import _native as native

    lib = native.library()
    probe = _host_state(1000, seed=6)
    limit = _static_limit(lib, native, probe)
    per_gaussian = 767
    assert limit % 64 == 0
    staging = 48 << 20  # CLAD3DGS_STATIC_STAGING_BYTES
    assert limit * per_gaussian <= staging
    assert (limit + 128) * per_gaussian > staging - 64 * 256
    n = limit + 1000  # two chunks: one full, one partial
    static_state = _host_state(n, seed=31)
    workspace_state = _host_state(n, seed=31)
    head, cfg, arrays, rates, b1, b2 = _arguments(*static_state, 1)
    status = lib.clad3dgs_gaussian_step_host_static(n, 3, *head, cfg, *arrays, rates,
                                                    b1, b2, limit + 64, 0)
    assert status == native.INVALID_ARGUMENT
    assert _identical(_snapshot(*static_state[:2]), _snapshot(*workspace_state[:2]))
    stream = torch.cuda.current_stream().cuda_stream
    status = lib.clad3dgs_gaussian_step_host_static(n, 3, *head, cfg, *arrays, rates,
                                                    b1, b2, limit, stream)
    assert status == native.OK, lib.clad3dgs_last_error()
    ws_chunk = 8192
    workspace = torch.empty(consume.host_step_workspace(ws_chunk), dtype=torch.uint8,
                            device=cuda)
    head, cfg, arrays, rates, b1, b2 = _arguments(*workspace_state, 1)
    status = lib.clad3dgs_gaussian_step_host(n, 3, *head, cfg, *arrays, rates, b1, b2,
                                             workspace.data_ptr(), workspace.numel(),
                                             ws_chunk, stream)
    assert status == native.OK, lib.clad3dgs_last_error()
    assert _identical(_snapshot(*static_state[:2]), _snapshot(*workspace_state[:2]))
