"""GPU parity of the Qwen3.5-MoE hybrid decoder (pokit_cuda_decoder_* with
arch POKIT_CUDA_ARCH_QWEN35MOE) against the reference's own Qwen35Runner on
benchmark configuration 3's model reduced to four layers: three Gated
DeltaNet layers and one gated full-attention layer, each followed by a MoE
block of 512 experts top-10 with the sigmoid-gated Q8_0 shared expert
(tests/golden/decoder_cfg3_L4.npz, made by tests/golden/make_decoder_golden.py
--arch qwen35 from the reference's generate_tokens and forward_token on a
synthetic GGUF; the weights are synthesised here in HBM from the same seeds).

Bar (north star): greedy token ids identical for the first 64 generated
tokens; the logits after the prompt within 1e-3 x their RMS.
"""
from pathlib import Path

import numpy as np
import pytest

from pokitlms_b200 import backend as B
from pokitlms_b200 import gguf

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "decoder_cfg3_L4.npz"


# Every layer (attention or DeltaNet) and its MoE block in one launch (the
# default); the full-attention layers as the fused attention block ahead of
# a separate MoE launch, and as three kernels; a DeltaNet layer and its MoE
# block as two launches, and the DeltaNet layer as the in-projection,
# conv1d, delta-step and ssm_out kernels.
MODES = {"attention_block": {}, "three_kernels": {"POKIT_CUDA_FUSED_ATTN": "0"},
         "attention_block_split": {"POKIT_CUDA_FUSED_ATTN_MOE": "0"},
         "delta_block": {"POKIT_CUDA_FUSED_DELTA_MOE": "0"},
         "delta_kernels": {"POKIT_CUDA_FUSED_DELTANET": "0"}}


@pytest.fixture(scope="module", params=list(MODES))
def decoder(cuda, request):
    g = np.load(GOLDEN)
    mp = pytest.MonkeyPatch()
    for k, v in MODES[request.param].items():
        mp.setenv(k, v)                      # read when the decoder is created
    try:
        dec = B.CudaDecoder(gguf.Qwen35MoeShape(layers=int(g["layers"])))
    finally:
        mp.undo()
    dec.synthesize_model()
    yield dec, g
    dec.close()


def _prefill_logits(dec, prompt):
    dec.reset()
    for i, t in enumerate(prompt[:-1]):
        assert dec.forward_token(int(t), i, logits=False) is None
    return dec.forward_token(int(prompt[-1]), len(prompt) - 1)


def test_logits_after_the_prompt_match_the_reference(decoder):
    dec, g = decoder
    logits = _prefill_logits(dec, g["prompt"])
    rms = float(g["logits_rms"])
    assert np.all(np.isfinite(logits))
    err_top = np.max(np.abs(logits[g["top_ids"]] - g["top_logits"]))
    err_sample = np.max(np.abs(logits[g["sample_pos"]] - g["sample_logits"]))
    assert err_top <= 1e-3 * rms and err_sample <= 1e-3 * rms, (err_top, err_sample, rms)
    assert int(np.argmax(logits)) == int(g["top_ids"][0])


def test_reset_clears_the_recurrent_state(decoder):
    dec, g = decoder
    first = _prefill_logits(dec, g["prompt"])
    second = _prefill_logits(dec, g["prompt"])             # reset zeroes conv and delta-rule states
    assert np.array_equal(first, second)


def test_greedy_tokens_match_the_reference(decoder):
    dec, g = decoder
    ids, stats = dec.generate_tokens(g["prompt"], len(g["ids"]))
    assert np.array_equal(ids[:64], g["ids"][:64])
    assert np.array_equal(ids, g["ids"])
    assert stats["generated_tokens"] == len(g["ids"]) and stats["decode_time_ns"] > 0
    again, _ = dec.generate_tokens(g["prompt"], 16)          # generate resets the state
    assert np.array_equal(again, g["ids"][:16])
    assert dec.step_graphs()[0] == 2


def test_each_layer_is_one_launch_by_default(decoder, request):
    """The default step: the embedding, one launch per layer (its mixer and
    its MoE block), the LM head and argmax when logits are wanted, and the
    position advance."""
    if request.node.callspec.params["decoder"] != "attention_block":
        pytest.skip("launch count of the default mode")
    dec, g = decoder
    layers = int(g["layers"])
    dec.generate_tokens(g["prompt"], 2)
    assert dec.launches_per_step() in (layers + 2, layers + 4)
