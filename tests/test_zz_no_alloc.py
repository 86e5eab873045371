"""GPU test of pokit_cuda_moe_forward_static_scratch, the MoE block entry
point for callers that cannot allocate device memory (their host framework
owns all of the GPU's memory, or they run on a thread that may not call
cudaMalloc).  It must give the same block output as the handle-based entry
point pokit_cuda_moe_forward, call after call, while its scratch lives in an
array compiled into the library.

The file name sorts last so that, in a run that stops at the first failure,
every other test has already run.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import cases
from pokitlms_b200 import backend as B
from pokitlms_b200 import synth
from pokitlms_b200._lib import (STATIC_SCRATCH_BYTES, ErrorBuffer, MoeBlockDevice,
                                STATUS_INVALID_ARGUMENT, STATUS_OK, lib)

pytestmark = pytest.mark.gpu


def _block(L, dev):
    return MoeBlockDevice(
        L.hidden, L.inter, L.experts, L.top_k, L.flavour, int(L.normalize),
        L.expert_weights_scale, dev["router"].data_ptr(), L.gate_type, L.up_type, L.down_type,
        dev["gate"].data_ptr(), dev["up"].data_ptr(), dev["down"].data_ptr(), 0, None, 8, 8, 8,
        None, None, None)


def _stream():
    s = torch.cuda.current_stream().cuda_stream
    return s if s else 0x1          # cudaStreamLegacy for torch's default stream


def test_static_scratch_matches_handle_entry_point(cuda):
    L = cases.moe_layer(hidden=1024, inter=512, experts=32, top_k=4, seed=21)
    dev = {k: torch.from_numpy(np.ascontiguousarray(getattr(L, k))).cuda()
           for k in ("router", "gate", "up", "down")}
    block = _block(L, dev)
    be = B.CudaMoeBackend(layers=1, hidden=L.hidden, inter=L.inter, experts=L.experts,
                          top_k=L.top_k)
    be.upload_layer(0, router=L.router, gate=L.gate, up=L.up, down=L.down,
                    ffn_norm=np.ones(L.hidden, np.float32))
    for call in range(2):                        # two calls in a row share the array
        x = torch.from_numpy(synth.activation(L.hidden, 21, call)).cuda()
        ref = torch.empty(L.hidden, device="cuda")
        ref_ids = torch.empty(L.top_k, dtype=torch.int32, device="cuda")
        be.forward(0, x, ref, ref_ids)
        be.synchronize()
        out = torch.full((L.hidden,), float("nan"), device="cuda")
        ids = torch.empty(L.top_k, dtype=torch.int32, device="cuda")
        w = torch.empty(L.top_k, device="cuda")
        err = ErrorBuffer()
        st = lib().pokit_cuda_moe_forward_static_scratch(
            C.byref(block), x.data_ptr(), out.data_ptr(), ids.data_ptr(), w.data_ptr(),
            _stream(), *err.args())
        assert st == STATUS_OK, err.text()
        torch.cuda.synchronize()
        r = ref.cpu().numpy().astype(np.float64)
        o = out.cpu().numpy()
        rms = float(np.sqrt(np.mean(r ** 2)))
        assert np.all(np.isfinite(o))
        assert float(np.max(np.abs(o - r))) <= 1e-3 * rms
        assert np.array_equal(ids.cpu().numpy(), ref_ids.cpu().numpy())
        assert abs(float(w.sum()) - 1.0) < 1e-5
    be.close()


def test_static_scratch_rejects_blocks_above_the_limit(cuda):
    L = cases.moe_layer(hidden=1024, inter=512, experts=32, top_k=4, seed=21)
    dev = {k: torch.from_numpy(np.ascontiguousarray(getattr(L, k))).cuda()
           for k in ("router", "gate", "up", "down")}
    block = _block(L, dev)
    block.inter = 8192                           # act of 5 slots x 8192 floats > the limit
    block.top_k = 64
    block.experts = 64
    out = torch.empty(L.hidden, device="cuda")
    x = torch.zeros(L.hidden, device="cuda")
    err = ErrorBuffer()
    st = lib().pokit_cuda_moe_forward_static_scratch(C.byref(block), x.data_ptr(),
                                                     out.data_ptr(), None, None, _stream(),
                                                     *err.args())
    assert st == STATUS_INVALID_ARGUMENT
    assert str(STATIC_SCRATCH_BYTES) in err.text()
