"""cpg_moe_forward_noalloc: the MoE block for callers that cannot allocate device memory where
they run it (an engine whose host program owns all device memory, a decode loop that may not
wait on the allocator). Its scratch is a fixed array
inside the library, so its output must match the workspace entry point's, call after call.

Collected last on purpose (file name), so a failure here cannot hide any other test."""
import ctypes

import numpy as np
import pytest

import oracle as O
from conftest import max_rel
from helpers import DECODE_TOL, device_layer

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _noalloc(lib, layer, x):
    T = x.shape[0]
    out = dict(mlp=torch.zeros((T, layer.d_model), dtype=torch.float32, device="cuda"),
               x_out=torch.empty_like(x),
               topk=torch.empty((T, layer.topk), dtype=torch.int32, device="cuda"),
               wt=torch.empty((T, layer.topk), dtype=torch.float32, device="cuda"),
               router=torch.empty((T, layer.n_experts), dtype=torch.float32, device="cuda"))
    rc = lib.cpg_moe_forward_noalloc(layer.handle, x.data_ptr(), None, T, out["mlp"].data_ptr(),
                                     out["x_out"].data_ptr(), out["topk"].data_ptr(), out["wt"].data_ptr(),
                                     out["router"].data_ptr(), torch.cuda.current_stream().cuda_stream)
    return rc, out


def test_noalloc_matches_workspace_entry_on_two_calls(orc):
    from cachepotato_b200 import _lib
    lib = _lib.lib()
    assert torch.cuda.is_available()
    D, F, E, K, T = 2048, 768, 128, 8, 64
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=808, oracle=orc)
    dl = device_layer(L)
    for call in range(2):
        x = torch.from_numpy(orc.normal(T * D, 900 + call, 1.0).reshape(T, D)).cuda()
        want = dl.forward(x)                                  # caller-workspace entry point
        rc, got = _noalloc(lib, dl, x)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.equal(got["topk"], want.topk_idx)
        assert max_rel(got["router"].cpu().numpy(), want.router.cpu().numpy()) <= 1e-5
        assert max_rel(got["wt"].cpu().numpy(), want.wt.cpu().numpy()) <= 1e-5
        assert max_rel(got["mlp"].cpu().numpy(), want.mlp.cpu().numpy()) <= DECODE_TOL
        assert max_rel(got["x_out"].cpu().numpy(), want.x_out.cpu().numpy()) <= DECODE_TOL


def test_noalloc_rejects_batches_beyond_its_scratch(orc):
    from cachepotato_b200 import _lib
    lib = _lib.lib()
    L = O.SynthLayer(256, 256, 16, 4, O.ENC_Q4, seed=809, oracle=orc)
    dl = device_layer(L)
    big = torch.zeros((4096, 256), dtype=torch.float32, device="cuda")
    rc, _ = _noalloc(lib, dl, big)
    assert rc == _lib.CPG_EINVAL and "scratch" in _lib.last_error()
