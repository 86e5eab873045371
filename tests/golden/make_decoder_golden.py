"""Golden greedy-decode targets of benchmark configurations 2 and 3 from the
reference's own decoders (test infrastructure; run in a container that has the
PokitLMs checkout).

Writes a reduced-layer synthetic Qwen3-30B-A3B-shaped GGUF (pokitlms_b200.gguf:
the configuration's shapes, vocabulary 151,936, Q4_K experts and attention,
Q6_K embedding and output, norms 1.0, expert_weights_norm = true), runs the
reference's Qwen3MoeRunner::generate_tokens on it through oracle/_ref/ref_runner
(built by `make -C oracle runner` from the reference's unmodified sources) with
a 32-token uniform-random prompt and 128 greedy tokens, and stores the prompt,
the generated ids and a compact view of the logits after the last prompt
token (their top 64 entries, and 4,096 entries at seeded positions, plus the
RMS of all of them) in tests/golden/decoder_cfg2_L{layers}.npz.  The GPU test
synthesises the same weights in HBM from the same seeds, so the 1.2 GB model
file is never committed or shipped.

With --arch qwen35 the model is configuration 3's Qwen3.5-MoE hybrid
(pokitlms_b200.gguf.Qwen35MoeShape: layer 3 full attention, the others Gated
DeltaNet; 512 experts top-10 with the Q8_0 shared expert, Q5_K/Q6_K down),
decoded by Qwen35Runner::generate_tokens, stored as decoder_cfg3_L{layers}.npz.

    python tests/golden/make_decoder_golden.py [--arch qwen3moe|qwen35] [--layers N] [--keep PATH]
"""
from __future__ import annotations

import argparse
import json
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from pokitlms_b200 import gguf  # noqa: E402

PROMPT_TOKENS, NEW_TOKENS, SAMPLE = 32, 128, 4096


def prompt_ids(vocab: int, seed: int = 0) -> np.ndarray:
    """The configuration's 32-token prompt of uniform random token ids."""
    return np.random.default_rng([seed, 0x7072]).integers(0, vocab, PROMPT_TOKENS, dtype=np.int64)


def logit_sample_positions(vocab: int) -> np.ndarray:
    return np.sort(np.random.default_rng([1, 0x6c73]).choice(vocab, SAMPLE, replace=False))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--arch", default="qwen3moe", choices=["qwen3moe", "qwen35"])
    ap.add_argument("--layers", type=int, default=None, help="default 2 (qwen3moe) or 4 (qwen35)")
    ap.add_argument("--keep", type=Path, default=None, help="keep the GGUF at this path")
    a = ap.parse_args()
    q35 = a.arch == "qwen35"
    layers = a.layers or (4 if q35 else 2)
    runner = ROOT / "oracle" / "_ref" / "ref_runner"
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "runner"], check=True)
    shape = gguf.Qwen35MoeShape(layers=layers) if q35 else gguf.Qwen3MoeShape(layers=layers)
    with tempfile.TemporaryDirectory() as tmp:
        model = a.keep or Path(tmp) / "model.gguf"
        (gguf.write_qwen35moe if q35 else gguf.write_qwen3moe)(model, shape)
        prompt = prompt_ids(shape.vocab)
        (Path(tmp) / "prompt.txt").write_text(" ".join(str(int(t)) for t in prompt))
        logits_file = Path(tmp) / "logits.bin"
        res = subprocess.run([str(runner)] + (["--qwen35"] if q35 else []) +
                             [str(model), str(Path(tmp) / "prompt.txt"), str(NEW_TOKENS), str(logits_file)],
                             capture_output=True, text=True, check=True)
        out = json.loads(res.stdout.strip().splitlines()[-1])
        logits = np.fromfile(logits_file, dtype=np.float32)
    ids = np.asarray(out["ids"], dtype=np.int64)
    top = np.argsort(-logits.astype(np.float64), kind="stable")[:64]
    pos = logit_sample_positions(shape.vocab)
    dest = ROOT / "tests" / "golden" / f"decoder_cfg{3 if q35 else 2}_L{layers}.npz"
    np.savez_compressed(dest, prompt=prompt, ids=ids, top_ids=top, top_logits=logits[top],
                        sample_pos=pos, sample_logits=logits[pos],
                        logits_rms=np.float64(np.sqrt(np.mean(logits.astype(np.float64) ** 2))),
                        layers=layers, decode_ns=out["decode_ns"], generated=out["generated"])
    print(f"{dest}: {len(ids)} ids, first 16 {ids[:16].tolist()}, distinct {len(set(ids.tolist()))}, "
          f"reference decode {out['generated'] / (out['decode_ns'] * 1e-9):.2f} tokens/s")


if __name__ == "__main__":
    main()
