"""GPU parity of the whole Qwen3-MoE decoder (pokit_cuda_decoder_*) against
the reference's own Qwen3MoeRunner on benchmark configuration 2's model
reduced to two layers (tests/golden/decoder_cfg2_L2.npz, made by
tests/golden/make_decoder_golden.py from the reference's generate_tokens and
forward_token on a synthetic GGUF; the weights are synthesised here in HBM
from the same seeds).

Bar (north star): greedy token ids identical for the first 64 generated
tokens; the logits after the prompt within 1e-3 x their RMS.  Every form of
the layer loop is checked (one chain launch for the whole loop, the fused
attention block beside the MoE chain, three attention kernels per layer).
"""
from pathlib import Path

import numpy as np
import pytest

from pokitlms_b200 import backend as B
from pokitlms_b200 import gguf

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "decoder_cfg2_L2.npz"


# The decoder's layer loop forms: the whole loop in one chain launch (the
# default), the fused attention block and the MoE chain as two launches per
# layer, and three attention kernels per layer.
MODES = {"layer_chain": {}, "attention_block": {"POKIT_CUDA_FUSED_LAYERS": "0"},
         "three_kernels": {"POKIT_CUDA_FUSED_LAYERS": "0", "POKIT_CUDA_FUSED_ATTN": "0"}}


@pytest.fixture(scope="module", params=list(MODES))
def decoder(cuda, request):
    g = np.load(GOLDEN)
    mp = pytest.MonkeyPatch()
    for k, v in MODES[request.param].items():
        mp.setenv(k, v)                      # read when the decoder is created
    try:
        dec = B.CudaDecoder(gguf.Qwen3MoeShape(layers=int(g["layers"])))
    finally:
        mp.undo()
    dec.synthesize_model()
    yield dec, g
    dec.close()


def test_logits_after_the_prompt_match_the_reference(decoder):
    dec, g = decoder
    prompt = g["prompt"]
    dec.reset()
    for i, t in enumerate(prompt[:-1]):
        assert dec.forward_token(int(t), i, logits=False) is None
    logits = dec.forward_token(int(prompt[-1]), len(prompt) - 1)
    rms = float(g["logits_rms"])
    assert np.all(np.isfinite(logits))
    err_top = np.max(np.abs(logits[g["top_ids"]] - g["top_logits"]))
    err_sample = np.max(np.abs(logits[g["sample_pos"]] - g["sample_logits"]))
    assert err_top <= 1e-3 * rms and err_sample <= 1e-3 * rms, (err_top, err_sample, rms)
    assert int(np.argmax(logits)) == int(g["top_ids"][0])


def test_greedy_tokens_match_the_reference(decoder):
    dec, g = decoder
    ids, stats = dec.generate_tokens(g["prompt"], len(g["ids"]))
    assert np.array_equal(ids[:64], g["ids"][:64])
    assert np.array_equal(ids, g["ids"])
    assert stats["generated_tokens"] == len(g["ids"]) and stats["decode_time_ns"] > 0
    again, _ = dec.generate_tokens(g["prompt"], 16)          # generate resets the state
    assert np.array_equal(again, g["ids"][:16])


def test_forward_token_argument_checks(decoder):
    dec, g = decoder
    dec.reset()
    with pytest.raises(ValueError):
        dec.forward_token(0, 3)                              # not the next position
    with pytest.raises(ValueError):
        dec.forward_token(dec.shape.vocab, 0)                # outside the vocabulary
    with pytest.raises(ValueError):
        dec.generate_tokens(g["prompt"], dec.shape.context)  # beyond the context
    dec.forward_token(int(g["prompt"][0]), 0, logits=False)  # the handle stays usable
