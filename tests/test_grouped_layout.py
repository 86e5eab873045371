"""CPU check of the grouped-expert GEMM's operand layout (pokit_grouped.cu).

Restates, in numpy, what the kernels put where:
  * the dequantiser's tensor-memory columns: column j = 32c + 4w + o holds
    the fp16 pair (low, high) of s_j * q for the Q4_K nibbles picked by one
    mask (and one 8-bit shift) of qs word w of chunk c;
  * pack_kernel's activation chunks: chunk 8c + w holds eight activations in
    the order that makes K element 2j + h of the activation operand meet the
    half h of column j;
  * the min operand: A = (m_0..m_7, m_0..m_7), B = (sub-block sums hi, lo);
and checks that d * (A . B) - dmin * (mins) reproduces the reference dot of
the decoded row (the oracle's decode of src/quantized_linear.cpp:166-205)
with every fp16 rounding the kernels make.
"""
import numpy as np

import cases
from oracle import oracle as O
from pokitlms_b200 import synth


def scales_mins(block):
    q = block[4:16].astype(np.uint32)
    sc = np.zeros(8, np.uint32)
    mn = np.zeros(8, np.uint32)
    for j in range(4):
        sc[j] = q[j] & 63
        mn[j] = q[j + 4] & 63
        sc[j + 4] = (q[j + 8] & 0xF) | ((q[j] >> 6) << 4)
        mn[j + 4] = (q[j + 8] >> 4) | ((q[j + 4] >> 6) << 4)
    return sc, mn


def fp16_fma(a, b, c):
    """One fp16 FMA (exact product and sum, one rounding to fp16)."""
    return np.float16(float(a) * float(b) + float(c))


def a_columns(block):
    """(128, 2) fp16 values of the tensor-memory columns for one superblock row,
    produced the way dequant_word does: low nibbles as 1024 + q times s minus
    1024 s, high nibbles masked in place as 1024 + 16 q times s / 16 minus 64 s."""
    sc, _ = scales_mins(block)
    qs = block[16:144]
    cols = np.zeros((128, 2), np.float16)
    for c in range(4):
        s_lo, s_hi = float(sc[2 * c]), float(sc[2 * c + 1])
        for w in range(8):
            W = int.from_bytes(bytes(qs[32 * c + 4 * w: 32 * c + 4 * w + 4]), "little")
            W8 = W >> 8
            for o, (word, mask) in enumerate([(W, 0x000F000F), (W8, 0x000F000F), (W, 0x00F000F0),
                                              (W8, 0x00F000F0)]):
                m = word & mask
                for h in range(2):
                    biased = 1024 + ((m >> (16 * h)) & 0xFF)      # fp16 bits 0x6400 | field
                    if mask == 0x000F000F:
                        cols[32 * c + 4 * w + o, h] = fp16_fma(biased, s_lo, -1024 * s_lo)
                    else:
                        cols[32 * c + 4 * w + o, h] = fp16_fma(biased, s_hi / 16, -64 * s_hi)
    return cols


def b_chunks(x):
    """(32, 8) activation chunks of one superblock (pack_kernel's order)."""
    xs = x.reshape(8, 32)
    out = np.zeros((32, 8), x.dtype)
    for c in range(4):
        for w in range(8):
            b0, b1 = xs[2 * c, 4 * w:4 * w + 4], xs[2 * c + 1, 4 * w:4 * w + 4]
            out[8 * c + w] = [b0[0], b0[2], b0[1], b0[3], b1[0], b1[2], b1[1], b1[3]]
    return out


def grouped_dot(block, x, split):
    """One superblock row . x the way the kernels compute it (float64 sums)."""
    d = float(np.frombuffer(bytes(block[0:2]), np.float16)[0])
    dmin = float(np.frombuffer(bytes(block[2:4]), np.float16)[0])
    _, mn = scales_mins(block)
    amax = float(np.max(np.abs(x)))
    ex = int(np.frexp(amax)[1]) if amax > 0 else 0
    sig = max(-100, min(100, ex - 10))
    xs = (x.astype(np.float64) * 2.0 ** -sig).astype(np.float32)   # exact power-of-two scaling
    hi = xs.astype(np.float16)
    lo = (xs - hi.astype(np.float32)).astype(np.float16)
    cols = a_columns(block).astype(np.float64)
    main = 0.0
    for part in ([hi, lo] if split else [hi]):
        bk = b_chunks(part.astype(np.float64)).reshape(-1)       # K order kappa = 0..255
        main += float(np.sum(cols[:, 0] * bk[0::2] + cols[:, 1] * bk[1::2]))
    sums = xs.reshape(8, 32).sum(axis=1, dtype=np.float32)
    s_hi = sums.astype(np.float16)
    s_lo = (sums - s_hi.astype(np.float32)).astype(np.float16)
    mins = float(np.sum(mn.astype(np.float64) * (s_hi.astype(np.float64) + s_lo.astype(np.float64))))
    return (d * main - dmin * mins) * 2.0 ** sig


def test_dequantised_columns_are_exact_scale_times_quant():
    blocks = synth.synth_blocks(cases.Q4_K, 16, seed=5, stream_id=1).reshape(16, 144)
    for b in range(16):
        sc, _ = scales_mins(blocks[b])
        cols = a_columns(blocks[b]).astype(np.float64)
        qs = blocks[b][16:144]
        for c in range(4):
            lo = (qs[32 * c:32 * c + 32] & 0xF).astype(np.float64) * sc[2 * c]
            hi = (qs[32 * c:32 * c + 32] >> 4).astype(np.float64) * sc[2 * c + 1]
            assert sorted(cols[32 * c:32 * c + 32][:, :].ravel()) == sorted(np.concatenate([lo, hi]))


def test_operand_layout_reproduces_q4k_dot():
    blocks = synth.synth_blocks(cases.Q4_K, 24, seed=7, stream_id=3).reshape(24, 144)
    rng = np.random.default_rng(1)
    for b in range(24):
        block = blocks[b]
        w = O.dequantize_row(cases.Q4_K, block, 256).astype(np.float64)
        # BF16 activations (exact in fp16 after scaling, no lo part) ...
        _, xb = synth.bf16_round(rng.standard_normal(256, dtype=np.float32))
        ref = float(np.dot(w, xb.astype(np.float64)))
        scale = float(np.sum(np.abs(w * xb)))
        assert abs(grouped_dot(block, xb, split=False) - ref) <= 1e-6 * scale
        # ... and F32 activations of any magnitude with the hi + lo split.
        xf = rng.standard_normal(256).astype(np.float32) * np.float32(10.0 ** rng.uniform(-3, 4))
        ref = float(np.dot(w, xf.astype(np.float64)))
        scale = float(np.sum(np.abs(w * xf)))
        assert abs(grouped_dot(block, xf, split=True) - ref) <= 1e-6 * scale


def test_single_fp16_part_is_not_enough_for_f32():
    """Why F32 activations carry a lo part: hi alone misses ~2^-12 per element."""
    blocks = synth.synth_blocks(cases.Q4_K, 8, seed=8, stream_id=3).reshape(8, 144)
    rng = np.random.default_rng(2)
    worst = 0.0
    for b in range(8):
        w = O.dequantize_row(cases.Q4_K, blocks[b], 256).astype(np.float64)
        xf = rng.standard_normal(256).astype(np.float32)
        ref = float(np.dot(w, xf.astype(np.float64)))
        scale = float(np.sum(np.abs(w * xf)))
        worst = max(worst, abs(grouped_dot(blocks[b], xf, split=False) - ref) / scale)
    assert worst > 1e-5


# ---------------------------------------------------------------------------
# Skinny tiles (thin_gemm_kernel): mma.sync.m16n8k16 fragments.
# ---------------------------------------------------------------------------

def pair_scales(hdr_words, t):
    """q4k_pair_scales: (scale, min) bytes of sub-blocks 2t, 2t + 1 without a
    branch on t, from the header's scale words hy, hz, hw."""
    hy, hz, hw = hdr_words
    sh = 16 * (t & 1)
    a, b, c = hy >> sh, hz >> sh, hw >> sh
    sc_lo, mn_lo = a & 0x3F3F, b & 0x3F3F
    sc_hi = (c & 0x0F0F) | ((a >> 2) & 0x3030)
    mn_hi = ((c >> 4) & 0x0F0F) | ((b >> 2) & 0x3030)
    sc, mn = (sc_hi, mn_hi) if t >= 2 else (sc_lo, mn_lo)
    return (sc & 0xFF, (sc >> 8) & 0xFF), (mn & 0xFF, (mn >> 8) & 0xFF)


def test_pair_scales_match_k_scale_min():
    rng = np.random.default_rng(11)
    for _ in range(500):
        block = np.zeros(144, np.uint8)
        block[4:16] = rng.integers(0, 256, 12, dtype=np.uint8)
        sc, mn = scales_mins(block)
        words = [int.from_bytes(bytes(block[4 + 4 * i:8 + 4 * i]), "little") for i in range(3)]
        for t in range(4):
            (s0, s1), (m0, m1) = pair_scales(words, t)
            assert (s0, s1, m0, m1) == (sc[2 * t], sc[2 * t + 1], mn[2 * t], mn[2 * t + 1])


THIN_TAIL, THIN_SEG, THIN_TOK = 288, 144, 576


def thin_chunk_offset(n, t, w):
    """pack_kernel's skinny placement: byte offset of token n's chunk w of lane
    quarter t within a superblock's hi (or lo) part."""
    return THIN_TAIL + n * THIN_TOK + t * THIN_SEG + 16 * w


def test_thin_reads_are_conflict_free_and_disjoint():
    """A quarter warp (tokens g = 0, 1 x lane quarters t = 0..3) reads chunk w
    of its (g, t) segment: eight distinct 16-byte bank groups; and no two
    chunks of the 8 x 4 x 8 overlap or spill past the part."""
    for w in range(8):
        for g0 in range(0, 8, 2):
            groups = {(thin_chunk_offset(g, t, w) // 16) % 8 for g in (g0, g0 + 1) for t in range(4)}
            assert len(groups) == 8
    offs = sorted(thin_chunk_offset(n, t, w) for n in range(8) for t in range(4) for w in range(8))
    assert all(b - a >= 16 for a, b in zip(offs, offs[1:]))
    assert offs[-1] + 16 <= THIN_TAIL + 8 * THIN_TOK


def thin_token_region(chunks, n):
    """One token's 32 chunks (8 fp16 each) placed as pack_kernel writes them,
    read back at the consumer's offsets."""
    mem = {}
    for t in range(4):
        for w in range(8):
            mem[thin_chunk_offset(n, t, w)] = chunks[8 * t + w]
    region = np.zeros((4, 8, 8), chunks.dtype)
    for t in range(4):
        for w in range(8):
            region[t, w] = mem[THIN_TAIL + n * THIN_TOK + t * THIN_SEG + (w << 4)]
    return region


def thin_dot(block, x, split, n=3):
    """One superblock row . x through the mma.sync fragments: thread (g, t)
    supplies, for qs word w and nibble parity h, A = dequant_word output
    2h + u (u = 0: logical k 2t, 2t+1; u = 1: k 2t+8, 2t+9) and B = the
    chunk's fp16 pair 2h + u read back from its packed place."""
    d = float(np.frombuffer(bytes(block[0:2]), np.float16)[0])
    dmin = float(np.frombuffer(bytes(block[2:4]), np.float16)[0])
    _, mn = scales_mins(block)
    amax = float(np.max(np.abs(x)))
    ex = int(np.frexp(amax)[1]) if amax > 0 else 0
    sig = max(-100, min(100, ex - 10))
    xs = (x.astype(np.float64) * 2.0 ** -sig).astype(np.float32)
    hi = xs.astype(np.float16)
    lo = (xs - hi.astype(np.float32)).astype(np.float16)
    cols = a_columns(block).astype(np.float64)          # dequant_word outputs, (128 columns, 2 halves)
    main = 0.0
    for part in ([hi, lo] if split else [hi]):
        region = thin_token_region(b_chunks(part), n)
        for t in range(4):
            for w in range(8):
                chunk = region[t, w].astype(np.float64)
                for h in range(2):
                    for u in range(2):
                        for e in range(2):
                            main += cols[32 * t + 4 * w + 2 * h + u, e] * chunk[4 * h + 2 * u + e]
    sums = xs.reshape(8, 32).sum(axis=1, dtype=np.float32)
    s_hi = sums.astype(np.float16).astype(np.float64)
    s_lo = (sums - s_hi.astype(np.float32)).astype(np.float16).astype(np.float64)
    # min MMA: a0 = a2 = (m_2t, m_2t+1), b0 = (hi_2t, hi_2t+1), b1 = (lo_2t, lo_2t+1)
    mins = sum(mn[2 * t + e] * (s_hi[2 * t + e] + s_lo[2 * t + e]) for t in range(4) for e in range(2))
    return (d * main - dmin * mins) * 2.0 ** sig


def test_thin_fragments_cover_every_k_once():
    seen = set()
    for t in range(4):
        for w in range(8):
            for h in range(2):
                for u in range(2):
                    for e in range(2):
                        j = 32 * t + 4 * w + 2 * h + u
                        seen.add((j, e, 8 * (8 * t + w) + 4 * h + 2 * u + e))
    # Each (column, half) meets chunk element 2 * (2j + half) ... exactly the tensor-core pairing.
    assert len(seen) == 256
    assert all(k == 2 * j + e for j, e, k in seen)


def test_thin_layout_reproduces_q4k_dot():
    blocks = synth.synth_blocks(cases.Q4_K, 12, seed=9, stream_id=4).reshape(12, 144)
    rng = np.random.default_rng(3)
    for b in range(12):
        block = blocks[b]
        w = O.dequantize_row(cases.Q4_K, block, 256).astype(np.float64)
        _, xb = synth.bf16_round(rng.standard_normal(256, dtype=np.float32))
        ref = float(np.dot(w, xb.astype(np.float64)))
        scale = float(np.sum(np.abs(w * xb)))
        assert abs(thin_dot(block, xb, split=False, n=b % 8) - ref) <= 1e-6 * scale
        xf = rng.standard_normal(256).astype(np.float32) * np.float32(10.0 ** rng.uniform(-3, 4))
        ref = float(np.dot(w, xf.astype(np.float64)))
        scale = float(np.sum(np.abs(w * xf)))
        assert abs(thin_dot(block, xf, split=True, n=b % 8) - ref) <= 1e-6 * scale


def group_tiles(counts, tile=64, skinny=8):
    """group_kernel's tile bookkeeping for per-expert pair counts: tile ids in
    expert order, and tile_order = the tiles of > skinny tokens, then the
    others, each at the position the kernel writes it to."""
    thin = [1 if (c % tile) and (c % tile) <= skinny else 0 for c in counts]
    ntiles = [(c + tile - 1) // tile for c in counts]
    off_tile = np.concatenate([[0], np.cumsum(ntiles)[:-1]]).astype(int)
    off_thin = np.concatenate([[0], np.cumsum(thin)[:-1]]).astype(int)
    total, n_thin = int(sum(ntiles)), int(sum(thin))
    large = total - n_thin
    order = [-1] * total
    sizes = {}
    for e, c in enumerate(counts):
        for i in range(ntiles[e]):
            t = off_tile[e] + i
            n = min(tile, c - i * tile)
            sizes[t] = n
            pos = large + off_thin[e] if n <= skinny else t - off_thin[e]
            assert 0 <= pos < total and order[pos] == -1, (e, i, pos)
            order[pos] = t
    return order, sizes, large


def test_tile_order_puts_large_tiles_first_as_a_permutation():
    rng = np.random.default_rng(12)
    for _ in range(300):
        E = int(rng.integers(1, 64))
        counts = [int(v) for v in rng.choice([0, 1, 3, 8, 9, 40, 63, 64, 65, 72, 73, 128, 200], size=E)]
        order, sizes, large = group_tiles(counts)
        assert sorted(order) == list(range(len(order)))
        assert all(sizes[t] > 8 for t in order[:large])
        assert all(sizes[t] <= 8 for t in order[large:])
        # within each list, tiles keep expert order (ids increase)
        assert order[:large] == sorted(order[:large]) and order[large:] == sorted(order[large:])
