"""A bounded device wait that runs out, on one GPU, without faulting it.

The fused cross-GPU sum polls every peer's exchange words with a bounded
number of polls (nsm_exchange_set_spin_limit).  Here a world-2 exchange is
connected inside one process and only rank 0 ever runs: rank 1's words are
never written, so rank 0's router gives up after the short limit, records
NSM_ERR_TIMEOUT in the workspace error word and returns.  The host reads that
status through nsm_workspace_error, and a normal decode on the same CUDA
context afterwards must still match the oracle -- the failure left the context
usable.  Only one rank's kernels are launched, so no two kernels on this GPU
wait on each other.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from next_step_ai_b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)


def _local_world2(lib, hidden):
    from next_step_ai_b200 import _lib

    exs = [ctypes.c_void_p(), ctypes.c_void_p()]
    for r in range(2):
        handle = (ctypes.c_char * _lib.NSM_IPC_HANDLE_BYTES)()
        _lib.check(lib.nsm_exchange_create(2, r, hidden, ctypes.byref(exs[r]), handle), "nsm_exchange_create")
    arr = (ctypes.c_void_p * 2)(exs[0].value, exs[1].value)
    _lib.check(lib.nsm_exchange_connect_local(arr, 2), "nsm_exchange_connect_local")
    return exs


@pytest.mark.parametrize("token_kernel", [False, True])
def test_exchange_wait_runs_out_and_the_context_survives(dev, token_kernel):
    """Both execution paths: the per-layer kernels (the router kernel waits)
    and the one-launch token kernel (its first phase waits; the other CTAs
    see the recorded error and leave too)."""
    from next_step_ai_b200 import _lib
    from next_step_ai_b200._torch import WORKSPACES
    from next_step_ai_b200.engine import SparseMlpDecoder
    from tests.test_gpu_engine import _build, _host_refs, _per_layer_check, _t

    lib = _lib.load()
    shape, layers, host = _build("small", 2, dev, seed=90)
    x0 = _t((np.random.default_rng(4).standard_normal(shape.hidden)).astype(np.float32), dev)
    dec = SparseMlpDecoder(layers, 3, token_kernel=token_kernel)
    torch.cuda.synchronize()

    def errors():
        return [dec.token_error()] if token_kernel else list(WORKSPACES.errors().values())

    errors()  # start from clear error words
    exs = _local_world2(lib, shape.hidden)
    try:
        _lib.check(lib.nsm_exchange_set_spin_limit(exs[0], 2000), "nsm_exchange_set_spin_limit")
        dec._ex = exs[0]  # rank 0 of a world of two whose rank 1 never runs
        dec.residual.copy_(x0)
        dec.step_eager()  # layers 1, 2 and the final flush each wait for rank 1 and give up
        torch.cuda.synchronize()
        errs = errors()
        assert _lib.NSM_ERR_TIMEOUT in errs, errs
        assert all(v == 0 for v in errors())  # the read cleared it
    finally:
        dec._ex = None
        torch.cuda.synchronize()
        for ex in exs:
            lib.nsm_exchange_destroy(ex)
    # the same context, the same workspace: a normal token matches the oracle
    route_ref, mlp_ref = _host_refs(shape, host)
    _per_layer_check(dec, x0, route_ref, mlp_ref, [host[i % 2][2] for i in range(3)])
    assert all(v == 0 for v in errors())


def test_wait_limit_settings_are_validated(dev):
    from next_step_ai_b200 import _lib

    lib = _lib.load()
    assert lib.nsm_exchange_set_spin_limit(None, 10) == _lib.NSM_ERR_INVALID_ARG
    prev = lib.nsm_set_copy_wait_limit(0)
    assert prev > 0
    assert lib.nsm_set_copy_wait_limit(-1) == _lib.NSM_ERR_INVALID_ARG
    assert lib.nsm_set_copy_wait_limit(prev) == prev
