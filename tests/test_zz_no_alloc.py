"""GPU test of pokit_cuda_moe_forward_static_scratch, the MoE block entry
point for callers that cannot allocate device memory (their host framework
owns all of the GPU's memory, or they run on a thread that may not call
cudaMalloc).  It must give the same block output as the handle-based entry
point pokit_cuda_moe_forward, call after call, while its scratch lives in an
array compiled into the library.

Cases: the all-Q4_K tensor-core block (eight activation replicas fit the
array), a Q4_K block whose activations leave room for fewer replicas (the
down kernel then spreads its reads over fewer copies), and the Qwen3.5
flavour with a Q8_0 shared expert and a Q6_K down projection (the generic
kernels).  The misaligned-router rejection needs no GPU (it is refused
before any CUDA call) and runs in the CPU suite too.

The file name sorts last so that, in a run that stops at the first failure,
every other test has already run.
"""
import ctypes as C

import numpy as np
import pytest

import cases
from pokitlms_b200 import backend as B
from pokitlms_b200 import synth
from pokitlms_b200._lib import (STATIC_SCRATCH_BYTES, ErrorBuffer, MoeBlockDevice,
                                STATUS_INVALID_ARGUMENT, STATUS_OK, lib)


def _block(L, ptr):
    sh = L.shared_inter or 0
    return MoeBlockDevice(
        L.hidden, L.inter, L.experts, L.top_k, L.flavour, int(L.normalize),
        L.expert_weights_scale, ptr["router"], L.gate_type, L.up_type, L.down_type,
        ptr["gate"], ptr["up"], ptr["down"], sh, ptr.get("shared_router"), 8, 8, 8,
        ptr.get("shared_gate"), ptr.get("shared_up"), ptr.get("shared_down"))


def _stream():
    import torch
    s = torch.cuda.current_stream().cuda_stream
    return s if s else 0x1          # cudaStreamLegacy for torch's default stream


TENSORS = ("router", "gate", "up", "down", "shared_router", "shared_gate", "shared_up", "shared_down")

CASES = {
    # hidden, inter, experts, top_k, flavour, down type, shared inter
    "q4k_tensor_core": dict(hidden=1024, inter=512, experts=32, top_k=4, seed=21),
    # 8 x 1536 activation floats per replica: only one or two replicas fit.
    "q4k_fewer_replicas": dict(hidden=1024, inter=1536, experts=32, top_k=8, seed=22),
    "qwen35_shared_q6k": dict(hidden=1024, inter=512, experts=32, top_k=4, seed=23, flavour=1,
                              down_type=cases.Q6_K, shared_inter=256, expert_weights_scale=2.5),
}


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CASES))
def test_static_scratch_matches_handle_entry_point(cuda, name):
    import torch
    L = cases.moe_layer(**CASES[name])
    dev = {k: torch.from_numpy(np.ascontiguousarray(getattr(L, k))).cuda()
           for k in TENSORS if getattr(L, k, None) is not None}
    block = _block(L, {k: v.data_ptr() for k, v in dev.items()})
    kw = dict(layers=1, hidden=L.hidden, inter=L.inter, experts=L.experts, top_k=L.top_k,
              flavour=L.flavour, expert_weights_scale=L.expert_weights_scale, down_type=L.down_type)
    if L.shared_inter:
        kw["shared_inter"] = L.shared_inter
    be = B.CudaMoeBackend(**kw)
    be.upload_layer(0, router=L.router, gate=L.gate, up=L.up, down=L.down,
                    ffn_norm=np.ones(L.hidden, np.float32), shared_router=L.shared_router,
                    shared_gate=L.shared_gate, shared_up=L.shared_up, shared_down=L.shared_down)
    for call in range(2):                        # two calls in a row share the array
        x = torch.from_numpy(synth.activation(L.hidden, 21, call)).cuda()
        ref = torch.empty(L.hidden, device="cuda")
        ref_ids = torch.empty(L.top_k, dtype=torch.int32, device="cuda")
        ref_w = torch.empty(L.top_k, device="cuda")
        be.forward(0, x, ref, ref_ids, ref_w)
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
        assert np.allclose(w.cpu().numpy(), ref_w.cpu().numpy(), rtol=1e-6, atol=0)
    be.close()


@pytest.mark.gpu
def test_static_scratch_rejects_blocks_above_the_limit(cuda):
    import torch
    L = cases.moe_layer(hidden=1024, inter=512, experts=32, top_k=4, seed=21)
    dev = {k: torch.from_numpy(np.ascontiguousarray(getattr(L, k))).cuda()
           for k in ("router", "gate", "up", "down")}
    block = _block(L, {k: v.data_ptr() for k, v in dev.items()})
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


def test_static_scratch_rejects_a_misaligned_router():
    """A router 4 bytes into a buffer would fault the kernels' 16-byte loads;
    the entry refuses it before touching a device (the addresses below are
    never dereferenced)."""
    from pokitlms_b200 import build
    build.build()
    base = 0x7f0000000000
    for field in ("router", "shared_router"):
        ptr = {k: base + i * 0x1000000 for i, k in enumerate(TENSORS)}
        ptr[field] += 4
        L = cases.MoeShape(hidden=1024, inter=512, experts=32, top_k=4, flavour=1, shared_inter=256)
        block = _block(L, ptr)
        err = ErrorBuffer()
        st = lib().pokit_cuda_moe_forward_static_scratch(C.byref(block), base, base + 0x100, None,
                                                         None, None, *err.args())
        assert st == STATUS_INVALID_ARGUMENT, err.text()
        assert "16-byte aligned" in err.text()
