"""GPU parity tests of the per-matrix kernels, called through the C ABI.

Tolerances:
  * the reference's own CPU/Vulkan parity cases keep the reference's bound,
    |gpu - cpu| <= 0.001 + 2e-5 * |cpu| (vulkan_linear_cases.hpp:81);
  * seeded benchmark-shaped matrices: max |gpu - cpu| <= 1e-4 * rms(cpu)
    (FP32 accumulation in a different order than the reference's sequential
    per-block dot; observed error is ~1e-6 relative);
  * dequantisation and routing ids: bit-exact.
"""
import numpy as np
import pytest
import torch

import cases
from oracle import oracle as O
from pokitlms_b200 import backend as B
from pokitlms_b200 import synth

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_linear(t, w, rows, cols, x, offset=0):
    wd = dev(np.concatenate([np.zeros(offset, dtype=np.uint8), w.view(np.uint8)]))
    wd = wd[offset:] if offset else wd
    y = torch.full((rows,), float("nan"), device="cuda")
    B.linear(t, wd, rows, cols, dev(x), y)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def assert_close_rms(got, ref, rel=1e-4):
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    err = float(np.max(np.abs(got.astype(np.float64) - ref)))
    assert np.all(np.isfinite(got))
    assert err <= rel * rms + 1e-6, (err, rms)


SHAPES = [(cases.Q4_K, 768, 2048), (cases.Q4_K, 2048, 768), (cases.Q4_K, 1536, 4096),
          (cases.Q4_K, 4096, 1536), (cases.Q4_K, 1, 256), (cases.Q4_K, 13, 512),
          (cases.Q5_K, 2048, 512), (cases.Q5_K, 37, 768), (cases.Q6_K, 2048, 512),
          (cases.Q6_K, 37, 768), (cases.Q6_K, 5, 2048), (cases.Q6_K, 16003, 2048),
          (cases.Q6_K, 300, 4096), (cases.Q8_0, 512, 2048),
          (cases.Q8_0, 2048, 512), (cases.Q8_0, 3, 32), (cases.F32, 128, 2048),
          (cases.F32, 1, 2048), (cases.F32, 37, 257)]


@pytest.mark.parametrize("t,rows,cols", SHAPES)
def test_linear_matches_oracle(cuda, t, rows, cols):
    if t == cases.F32:
        w = np.random.default_rng(rows).standard_normal(rows * cols).astype(np.float32)
    else:
        w = synth.synth_matrix(t, rows, cols, 5, rows)
    x = synth.activation(cols, 5, rows)
    ref = O.linear(t, x, w, rows)
    assert_close_rms(run_linear(t, w, rows, cols, x), ref)


@pytest.mark.parametrize("rows,cols", [(768, 2048), (37, 512), (2048, 768)])
def test_q4k_fast_and_generic_paths_agree(cuda, rows, cols):
    """A 16-byte-aligned Q4_K matrix takes the 128-bit chunk path; the same
    bytes at a 2-byte offset take the staged generic path."""
    w = synth.synth_matrix(cases.Q4_K, rows, cols, 8, 1)
    x = synth.activation(cols, 8)
    ref = O.linear(cases.Q4_K, x, w, rows)
    fast = run_linear(cases.Q4_K, w, rows, cols, x)
    generic = run_linear(cases.Q4_K, w, rows, cols, x, offset=2)
    assert_close_rms(fast, ref)
    assert_close_rms(generic, ref)


@pytest.mark.parametrize("rows,cols", [(777, 2048), (3001, 4096)])
def test_q6k_tensor_and_row_paths_agree(cuda, rows, cols):
    """A 16-byte-aligned Q6_K matrix of 2048k columns takes the integer
    tensor-core kernel (persistent, several 16-row tiles per CTA); the same
    bytes at a 2-byte offset take the FP32 path."""
    w = synth.synth_matrix(cases.Q6_K, rows, cols, 9, 2)
    x = synth.activation(cols, 9)
    ref = O.linear(cases.Q6_K, x, w, rows)
    assert_close_rms(run_linear(cases.Q6_K, w, rows, cols, x), ref)
    assert_close_rms(run_linear(cases.Q6_K, w, rows, cols, x, offset=2), ref)


def test_reference_parity_cases(cuda):
    """vulkan_linear_cases.hpp:31-90 inputs, tolerance and repeats."""
    checked = 0
    for t, rows, cols, payload, inp in cases.vulkan_parity_cases():
        if t not in (cases.F32, cases.Q8_0, cases.Q4_K, cases.Q5_K, cases.Q6_K):
            continue
        x = inp
        for _ in range(3):
            cpu = O.linear(t, x, payload, rows)
            gpu = run_linear(t, payload, rows, cols, x)
            err = np.abs(cpu.astype(np.float64) - gpu)
            assert np.all(np.isfinite(gpu))
            assert np.all(err <= 0.001 + 0.00002 * np.abs(cpu)), (t, float(err.max()))
            x = (x * np.float32(-0.75)).astype(np.float32)
        checked += 1
    assert checked == 5


@pytest.mark.parametrize("t,rows,cols", [(cases.Q4_K, 64, 2048), (cases.Q5_K, 64, 512),
                                         (cases.Q6_K, 64, 768), (cases.Q8_0, 64, 2048)])
def test_dequantize_bit_exact(cuda, t, rows, cols):
    w = synth.synth_matrix(t, rows, cols, 2, 2)
    out = torch.empty(rows * cols, device="cuda")
    B.dequantize_rows(t, dev(w), rows, cols, out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    rb = O.row_bytes(t, cols)
    ref = np.concatenate([O.dequantize_row(t, w[r * rb:(r + 1) * rb], cols) for r in range(rows)])
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("builder,t", [(cases.q4k_known_answer_block, cases.Q4_K),
                                       (cases.q6k_known_answer_block, cases.Q6_K),
                                       (cases.q8_0_known_answer_block, cases.Q8_0),
                                       (lambda: cases.q5k_known_answer_blocks()[0], cases.Q5_K),
                                       (lambda: cases.q5k_known_answer_blocks()[1], cases.Q5_K)])
def test_known_answer_blocks(cuda, builder, t):
    block, expected = builder()
    n = expected.size
    out = torch.empty(n, device="cuda")
    B.dequantize_rows(t, dev(block), 1, n, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), expected)
    x = cases.check_block_input()[:n]
    y = run_linear(t, block, 1, n, x)[0]
    assert abs(float(y) + 0.75 - (0.75 + float(np.dot(x.astype(np.float64), expected)))) < 0.01


@pytest.mark.parametrize("flavour", [0, 1])
@pytest.mark.parametrize("E,k", [(128, 8), (512, 10), (8, 8), (64, 1)])
def test_route_experts_matches_oracle(cuda, flavour, E, k):
    rng = np.random.default_rng(E * 10 + k)
    for trial in range(4):
        logits = rng.standard_normal(E).astype(np.float32) * np.float32(3.0)
        if trial == 3:
            logits[E // 2] = logits[E // 3] = logits.max()     # a tie at the top
        ids = torch.empty(k, dtype=torch.int32, device="cuda")
        w = torch.empty(k, device="cuda")
        B.route_experts(dev(logits), k, flavour, True, ids, w, expert_weights_scale=1.0)
        torch.cuda.synchronize()
        ref_ids, ref_p = O.route(flavour, logits, k)
        assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ref_ids)
        assert np.allclose(w.cpu().numpy(), ref_p, rtol=2e-6, atol=0)


def test_route_experts_scale_and_non_finite(cuda):
    logits = np.linspace(-1, 1, 32).astype(np.float32)
    ids = torch.empty(4, dtype=torch.int32, device="cuda")
    w = torch.empty(4, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    B.route_experts(dev(logits), 4, 1, True, ids, w, expert_weights_scale=2.5, status=status)
    torch.cuda.synchronize()
    ref_ids, ref_p = O.route(1, logits, 4)
    assert np.allclose(w.cpu().numpy(), ref_p * np.float32(2.5), rtol=2e-6)
    assert int(status.item()) == 0
    logits[7] = np.nan
    B.route_experts(dev(logits), 4, 0, True, ids, w, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 1
    assert sorted(ids.cpu().tolist()) == [0, 1, 2, 3] and float(w.abs().sum()) == 0.0


@pytest.mark.parametrize("t", [cases.Q4_K, cases.Q5_K, cases.Q6_K, cases.Q8_0])
def test_device_synthesis_matches_host(cuda, t):
    n = 1001
    bb = O.BLOCK[t][1]
    buf = torch.zeros(n * bb, dtype=torch.uint8, device="cuda")
    B.synthesize_blocks(t, 42, 17, n, buf)
    torch.cuda.synchronize()
    assert np.array_equal(buf.cpu().numpy(), synth.synth_blocks(t, n, 42, 17))


def test_linear_backend_host_spans(cuda):
    be = B.CudaLinearBackend(0)
    w = synth.synth_matrix(cases.Q4_K, 768, 2048, 3, 3)
    out = np.empty(768, dtype=np.float32)
    for rep in range(3):
        x = synth.activation(2048, 3, rep)
        assert be.try_linear(cases.Q4_K, w, 768, 2048, x, out)
        assert_close_rms(out, O.linear(cases.Q4_K, x, w, 768))
    w8 = synth.synth_matrix(cases.Q8_0, 64, 512, 3, 4)
    out8 = np.empty(64, dtype=np.float32)
    x8 = synth.activation(512, 3)
    assert be.try_linear(cases.Q8_0, w8, 64, 512, x8, out8)
    assert_close_rms(out8, O.linear(cases.Q8_0, x8, w8, 64))
    # Unsupported GGML type: not handled, caller falls back (tensor_linear.hpp:14).
    assert not be.try_linear(2, np.zeros(18 * 4, dtype=np.uint8), 4, 32,
                             np.zeros(32, dtype=np.float32), np.empty(4, dtype=np.float32))
    with pytest.raises(ValueError):
        be.try_linear(cases.Q4_K, w[:-1], 768, 2048, x, out)
    s = be.stats()
    assert s["linear_calls"] == 4 and s["dispatches"] == 4 and s["q4_k_dispatches"] == 3
    assert s["q8_0_dispatches"] == 1
    assert s["model_cache_uploaded_bytes"] == 0          # unkeyed calls stream, cache nothing
    be.close()


def test_linear_backend_reused_host_buffer_gets_the_new_weights(cuda):
    """The caller frees a matrix and the next one of the same size lands at
    the same host address (gate and up of an expert are both 884,736 B): the
    second call must see the second matrix's bytes."""
    be = B.CudaLinearBackend(0)
    buf = np.empty(768 * 8 * 144, dtype=np.uint8)
    out = np.empty(768, dtype=np.float32)
    x = synth.activation(2048, 5)
    for sid in (11, 12, 13):
        buf[:] = synth.synth_matrix(cases.Q4_K, 768, 2048, 5, sid)
        assert be.try_linear(cases.Q4_K, buf, 768, 2048, x, out)
        assert_close_rms(out, O.linear(cases.Q4_K, x, buf, 768))
    be.close()


def test_linear_backend_keyed_cache(cuda):
    be = B.CudaLinearBackend(0)
    w1 = synth.synth_matrix(cases.Q4_K, 256, 1024, 6, 1)
    w2 = synth.synth_matrix(cases.Q4_K, 256, 1024, 6, 2)
    x = synth.activation(1024, 6)
    out = np.empty(256, dtype=np.float32)
    assert be.try_linear(cases.Q4_K, w1, 256, 1024, x, out, key=1)
    assert_close_rms(out, O.linear(cases.Q4_K, x, w1, 256))
    assert be.try_linear(cases.Q4_K, w2, 256, 1024, x, out, key=2)
    assert_close_rms(out, O.linear(cases.Q4_K, x, w2, 256))
    s = be.stats()
    assert s["model_cache_uploaded_bytes"] == 2 * w1.nbytes
    assert s["model_cache_capacity_bytes"] == 2 * w1.nbytes
    # A cached key answers from HBM (its host bytes are not read again).
    assert be.try_linear(cases.Q4_K, w2, 256, 1024, x, out, key=1)
    assert_close_rms(out, O.linear(cases.Q4_K, x, w1, 256))
    # forget: the next call with the key uploads the new bytes.
    assert be.forget(1) and not be.forget(1)
    assert be.try_linear(cases.Q4_K, w2, 256, 1024, x, out, key=1)
    assert_close_rms(out, O.linear(cases.Q4_K, x, w2, 256))
    # A key reused for another shape is refused.
    with pytest.raises(ValueError):
        be.try_linear(cases.Q4_K, w1[: 128 * 4 * 144], 128, 1024, x, out[:128], key=2)
    # Capacity bounds the cache: least recently used entries go first.
    be.set_cache_capacity(w1.nbytes)
    assert be.stats()["model_cache_capacity_bytes"] == w1.nbytes
    be.try_linear(cases.Q4_K, w1, 256, 1024, x, out, key=3)
    assert be.stats()["model_cache_capacity_bytes"] == w1.nbytes
    assert_close_rms(out, O.linear(cases.Q4_K, x, w1, 256))
    be.close()
