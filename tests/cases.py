"""Shared test inputs: the reference's known-answer blocks and parity cases,
restated as generators, plus the benchmark-shaped MoE layers.

Sources (PokitLMs, paths relative to its project root):
  * Q5_K known-answer blocks: tests/regression_test.cpp:31-46 (check_block),
    :75-84 (pack_scale_min), :86-112 (test_q5_k).
  * Random-block parity cases: tests/vulkan_linear_cases.hpp:16-90
    (xorshift32 seed 0x5935a3b, 37 rows, 512 columns, scales pinned to fp16
    0x2800 / 0x2400, tolerance 0.001 + 2e-5 * |cpu|, 3 repeats with the input
    scaled by -0.75).
  * Q4_K / Q6_K / Q8_0 known-answer blocks: not in the reference (it pins them
    only through CPU/Vulkan parity); built here from the block layouts of
    src/quantized_linear.cpp:166-205, :330-358 and :387-423.
"""
from __future__ import annotations

import numpy as np

F32, Q8_0, Q4_K, Q5_K, Q6_K = 0, 8, 12, 13, 14
F16_TYPE, BF16_TYPE, Q4_0, Q4_1 = 1, 30, 2, 3


def u16(block: np.ndarray, offset: int, value: int) -> None:
    block[offset] = value & 255
    block[offset + 1] = value >> 8


def check_block_input() -> np.ndarray:
    """input[i] = ((i * 7) % 13 - 6) / 8 (regression_test.cpp:40)."""
    i = np.arange(256)
    return (((i * 7) % 13 - 6) / 8.0).astype(np.float32)


def pack_scale_min(block: np.ndarray, group: int, scale: int, minimum: int) -> None:
    """6-bit scale/min packing shared by Q4_K and Q5_K (regression_test.cpp:75-84)."""
    if group < 4:
        block[4 + group] |= scale
        block[8 + group] |= minimum
    else:
        block[group] |= (scale >> 4) << 6
        block[4 + group] |= (minimum >> 4) << 6
        block[8 + group] |= (scale & 15) | ((minimum & 15) << 4)


def q5k_known_answer_blocks() -> list[tuple[np.ndarray, np.ndarray]]:
    """The two Q5_K blocks of test_q5_k (regression_test.cpp:86-112) with their
    exact expected decodes."""
    out = []
    block = np.zeros(176, dtype=np.uint8)
    u16(block, 0, 0x3C00)                      # d = 1
    for g in range(8):
        pack_scale_min(block, g, 1, 0)
    block[48:] = 0x11
    out.append((block.copy(), np.ones(256, dtype=np.float32)))

    block = np.zeros(176, dtype=np.uint8)
    expected = np.zeros(256, dtype=np.float32)
    u16(block, 0, 0x3800)                      # d = 0.5
    u16(block, 2, 0x3400)                      # dmin = 0.25
    for g in range(8):
        scale = (g * 9 + 5) % 64
        minimum = (g * 11 + 7) % 64
        pack_scale_min(block, g, scale, minimum)
        for lane in range(32):
            index = g * 32 + lane
            quant = (index * 13 + g) % 32
            block[16 + lane] |= (quant >> 4) << g
            block[48 + (g // 2) * 32 + lane] |= (quant & 15) << (4 * (g % 2))
            expected[index] = np.float32(0.5) * np.float32(scale) * np.float32(quant) - \
                np.float32(0.25) * np.float32(minimum)
    out.append((block, expected))
    return out


def q4k_known_answer_block() -> tuple[np.ndarray, np.ndarray]:
    """A Q4_K block with every sub-block scale/min and nibble distinct
    (decode_q4_k layout: sub-block 2c takes the low nibbles of qs[32c..32c+31],
    sub-block 2c+1 the high nibbles)."""
    block = np.zeros(144, dtype=np.uint8)
    expected = np.zeros(256, dtype=np.float32)
    u16(block, 0, 0x3800)                      # d = 0.5
    u16(block, 2, 0x3400)                      # dmin = 0.25
    for g in range(8):
        scale = (g * 23 + 3) % 64
        minimum = (g * 29 + 11) % 64
        pack_scale_min(block, g, scale, minimum)
        chunk, part = divmod(g, 2)
        for i in range(32):
            quant = (i * 5 + g * 3) % 16
            block[16 + chunk * 32 + i] |= quant << (4 * part)
            ds = np.float32(0.5) * np.float32(scale)
            dm = np.float32(0.25) * np.float32(minimum)
            expected[g * 32 + i] = ds * np.float32(quant) - dm
    return block, expected


def q6k_known_answer_block() -> tuple[np.ndarray, np.ndarray]:
    """A Q6_K block with signed scales and all 64 quant levels (decode_q6_k:
    weight base+l+32j uses ql nibble (j>>1) of ql[l + 32(j&1)], qh bits 2j..2j+1
    of qh[l], scale scales[8h + l/16 + 2j]; value d * scale * (q - 32))."""
    block = np.zeros(210, dtype=np.uint8)
    expected = np.zeros(256, dtype=np.float32)
    u16(block, 208, 0x3000)                    # d = 0.125
    scales = [((s * 37 + 5) % 200) - 100 for s in range(16)]
    block[192:208] = np.array(scales, dtype=np.int8).view(np.uint8)
    for half in range(2):
        for j in range(4):
            for l in range(32):
                q = (l * 7 + j * 13 + half * 29) % 64
                ql_index = half * 64 + l + 32 * (j & 1)
                block[ql_index] |= (q & 15) << (4 * (j >> 1))
                block[128 + half * 32 + l] |= (q >> 4) << (2 * j)
                s = scales[half * 8 + l // 16 + 2 * j]
                expected[half * 128 + 32 * j + l] = (np.float32(0.125) * np.float32(s)) * \
                    np.float32(q - 32)
    return block, expected


def q8_0_known_answer_block() -> tuple[np.ndarray, np.ndarray]:
    """A Q8_0 block: fp16 d then 32 int8 quants; value d * q."""
    block = np.zeros(34, dtype=np.uint8)
    u16(block, 0, 0x2C00)                      # d = 0.0625
    q = np.array([((i * 19) % 255) - 127 for i in range(32)], dtype=np.int8)
    block[2:] = q.view(np.uint8)
    expected = (np.float32(0.0625) * q.astype(np.float32)).astype(np.float32)
    return block, expected


class XorShift32:
    """The parity tests' generator, vulkan_linear_cases.hpp:18-22."""

    def __init__(self, state: int = 0x5935A3B):
        self.state = state

    def __call__(self) -> int:
        s = self.state
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        self.state = s
        return s


def vulkan_parity_cases():
    """Yields (type, rows, columns, payload uint8, input f32) in the order and
    with the random stream of one pass of vulkan_linear_cases.hpp:31-72.  Types
    this backend does not accelerate (F16, BF16, Q4_0, Q4_1) are generated and
    yielded too so the stream stays aligned; callers skip them."""
    rnd = XorShift32()
    for t in (F32, F16_TYPE, BF16_TYPE, Q4_0, Q4_1, Q8_0, Q4_K, Q5_K, Q6_K):
        columns = 257 if t in (F32, F16_TYPE, BF16_TYPE) else 512
        rows = 37
        block = 256 if (t >= 12 and t != BF16_TYPE) else 32
        nbytes = {Q4_0: 18, Q4_1: 20, Q8_0: 34, Q4_K: 144, Q5_K: 176}.get(t, 210)
        if t == F32:
            row_bytes = columns * 4
        elif t in (F16_TYPE, BF16_TYPE):
            row_bytes = columns * 2
        else:
            row_bytes = columns // block * nbytes
        payload = np.array([rnd() & 255 for _ in range(rows * row_bytes)], dtype=np.uint8)
        if t == F32:
            vals = np.array([((rnd() % 2049) - 1024) / 1024.0 for _ in range(rows * columns)],
                            dtype=np.float32)
            payload = vals.view(np.uint8).copy()
        elif t in (F16_TYPE, BF16_TYPE):
            halves = np.empty(rows * columns, dtype=np.uint16)
            for i in range(rows * columns):
                bits = 0x3400 + (rnd() & 0x3FF) if t == F16_TYPE else 0x3E80 + (rnd() & 0x7F)
                halves[i] = bits | (rnd() & 0x8000)
            payload = halves.view(np.uint8).copy()
        else:
            for r in range(rows):
                for b in range(columns // block):
                    off = r * row_bytes + b * nbytes
                    u16(payload, off + (208 if t == Q6_K else 0), 0x2800)
                    if t in (Q4_1, Q4_K, Q5_K):
                        u16(payload, off + 2, 0x2400)
        inp = np.array([((rnd() % 2049) - 1024) / 1024.0 for _ in range(columns)],
                       dtype=np.float32)
        yield t, rows, columns, payload, inp


def moe_layer(hidden=2048, inter=768, experts=128, top_k=8, seed=0, layer=0, flavour=0,
              down_type=Q4_K, shared_inter=0, expert_weights_scale=1.0, with_norm=False):
    """A benchmark-shaped MoE block built from the seeded synthetic generator
    (config 1 by default: hidden 2048, 128 experts top-8, inter 768, Q4_K)."""
    from oracle.oracle import MoeLayer
    from pokitlms_b200 import synth

    sid = lambda t: synth.stream_id(layer, t)  # noqa: E731
    L = MoeLayer(
        hidden=hidden, inter=inter, experts=experts, top_k=top_k,
        router=synth.router_weights(experts, hidden, seed, layer),
        gate=synth.synth_matrix(Q4_K, experts * inter, hidden, seed, sid(1)),
        up=synth.synth_matrix(Q4_K, experts * inter, hidden, seed, sid(2)),
        down=synth.synth_matrix(down_type, experts * hidden, inter, seed, sid(3)),
        down_type=down_type, flavour=flavour, normalize=True,
        expert_weights_scale=expert_weights_scale)
    if with_norm:
        L.ffn_norm = np.ones(hidden, dtype=np.float32)
    if shared_inter:
        L.shared_inter = shared_inter
        L.shared_router = synth.router_weights(1, hidden, seed, 1000 + layer)[0]
        L.shared_gate = synth.synth_matrix(Q8_0, shared_inter, hidden, seed, sid(6))
        L.shared_up = synth.synth_matrix(Q8_0, shared_inter, hidden, seed, sid(7))
        L.shared_down = synth.synth_matrix(Q8_0, hidden, shared_inter, seed, sid(8))
    return L


def route_margin(logits: np.ndarray, k: int) -> float:
    """Gap between the k-th and (k+1)-th largest logits (routing is only
    required to match where it exceeds 1e-5)."""
    s = np.sort(np.asarray(logits, dtype=np.float64))[::-1]
    return float(s[k - 1] - s[k]) if k < s.size else float("inf")


class MoeShape:
    """The shape and type fields of a MoE block without its tensors (for
    argument-validation tests that never reach a kernel)."""

    def __init__(self, hidden, inter, experts, top_k, flavour=0, shared_inter=0,
                 gate_type=Q4_K, up_type=Q4_K, down_type=Q4_K, normalize=True,
                 expert_weights_scale=1.0):
        self.hidden, self.inter, self.experts, self.top_k = hidden, inter, experts, top_k
        self.flavour, self.shared_inter = flavour, shared_inter
        self.gate_type, self.up_type, self.down_type = gate_type, up_type, down_type
        self.normalize, self.expert_weights_scale = normalize, expert_weights_scale


# Benchmark configuration 3's Gated DeltaNet mixer: 16 key heads, 32 value
# heads, head_dim 128, causal conv1d kernel 4, F32 recurrent state.
DELTA_NET_CFG3 = dict(key_heads=16, value_heads=32, key_dim=128, value_dim=128, conv_kernel=4, rms_epsilon=1e-6)


def delta_net_inputs(shape: dict, seed: int, steps: int):
    """Seeded synthetic inputs of the DeltaNet mixer: per step the projected
    q|k|v ~N(0,1) (x4), gate z ~N(0,1), alpha ~N(0,1), beta ~N(0,1); tensors
    conv1d weights ~N(0,0.5), ssm_a = -exp(N(0,0.5)) (the GGUF stores -exp(A_log)),
    dt_bias ~N(0,0.5), ssm_norm ~U(0.5,1.5)."""
    rng = np.random.default_rng([seed, 0x646e])
    kh, vh, dk, dv, K = (shape[k] for k in ("key_heads", "value_heads", "key_dim", "value_dim", "conv_kernel"))
    C = 2 * kh * dk + vh * dv
    f = lambda *s_, scale=1.0: (rng.standard_normal(s_, dtype=np.float32) * np.float32(scale))  # noqa: E731
    tensors = dict(conv_w=f(C, K, scale=0.5), a=-np.exp(f(vh, scale=0.5)).astype(np.float32),
                   dt_bias=f(vh, scale=0.5), norm=rng.uniform(0.5, 1.5, dv).astype(np.float32))
    steps_in = [dict(projected=f(C, scale=4.0), gate=f(vh * dv), alpha=f(vh), beta=f(vh)) for _ in range(steps)]
    return tensors, steps_in
