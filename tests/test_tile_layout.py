"""CPU emulation of the fragment-tile layout and of the tensor-core matvec's
lane arithmetic (laicompute_b200/csrc/tiles.cuh, mma_matvec.cuh, and the one-sequence
integer variant of mv_streamk.cuh).

The repack, the per-lane decode (bit tricks evaluated in binary16 with numpy),
the activation hi/lo split in fragment order and the mma.m16n8k16 operand
fragments are replayed here and must give W @ x of the dequantised weights.
"""
import numpy as np
import pytest

from laicompute_b200 import gguf, synth
from oracle import oracle as O

QB = {gguf.Q4_0: 256, gguf.Q8_0: 512, gguf.F16: 1024}
SRC = {gguf.Q4_0: 18, gguf.Q8_0: 34, gguf.F16: 64}


def frag_pos(k):
    return 2 * k if k < 4 else 2 * (k - 4) + 1


def elem_offset(t_, nb, r, i):
    t, rr = r >> 4, r & 15
    g, h = rr & 7, rr >> 3
    b, o = i >> 5, i & 31
    cc, k = o >> 3, o & 7
    chunk = (t * nb + b) * QB[t_]
    L = g * 4 + cc
    if t_ == gguf.Q4_0:
        return chunk + L * 8 + h * 4 + (k >> 1)
    if t_ == gguf.Q8_0:
        return chunk + L * 16 + h * 8 + frag_pos(k)
    return chunk + L * 32 + h * 16 + frag_pos(k) * 2


def scale_offset(nb, r, b):
    t, rr = r >> 4, r & 15
    return (t * nb + b) * 32 + (rr & 7) * 4 + (rr >> 3) * 2


def repack(t_, raw, rows, nb):
    """Port of repack_tiles_kernel."""
    ntiles = (rows + 15) // 16
    q = np.zeros(ntiles * nb * QB[t_], np.uint8)
    s = np.zeros(ntiles * nb * 32, np.uint8)
    raw = raw.reshape(rows, nb, SRC[t_])
    for r in range(rows):
        for b in range(nb):
            sp = raw[r, b]
            if t_ == gguf.F16:
                for o in range(32):
                    off = elem_offset(t_, nb, r, b * 32 + o)
                    q[off:off + 2] = sp[2 * o:2 * o + 2]
                continue
            so = scale_offset(nb, r, b)
            s[so:so + 2] = sp[0:2]
            if t_ == gguf.Q8_0:
                for o in range(32):
                    q[elem_offset(t_, nb, r, b * 32 + o)] = sp[2 + o]
            else:
                for j in range(16):
                    q[elem_offset(t_, nb, r, b * 32 + 2 * j)] = sp[2 + j]
    return q, s


def h(bits):
    return np.array([bits], dtype=np.uint16).view(np.float16)[0]


def h2(u32):
    """uint32 -> (low half, high half) as float16."""
    return h(u32 & 0xFFFF), h((u32 >> 16) & 0xFFFF)


def decode_q4(w):
    M = 0x64006400
    out = []
    for sh, kind in ((0, "lo"), (0, "hi"), (8, "lo"), (8, "hi")):
        ww = w >> sh
        if kind == "lo":
            a, b = h2((ww & 0x000F000F) | M)
            out.append((np.float16(a - np.float16(1032)), np.float16(b - np.float16(1032))))
        else:
            a, b = h2((ww & 0x00F000F0) | M)
            out.append((np.float16(np.float32(a) * np.float32(1 / 16) - 72),
                        np.float16(np.float32(b) * np.float32(1 / 16) - 72)))
    return out


def byte_perm(x, y, sel):
    src = [(x >> (8 * i)) & 0xFF for i in range(4)] + [(y >> (8 * i)) & 0xFF for i in range(4)]
    return sum(src[(sel >> (4 * i)) & 7] << (8 * i) for i in range(4))


def decode_q8(u0, u1):
    C, out = 0x64646464, []
    u0 ^= 0x80808080
    u1 ^= 0x80808080
    for u, sel in ((u0, 0x4140), (u0, 0x4342), (u1, 0x4140), (u1, 0x4342)):
        a, b = h2(byte_perm(u, C, sel))
        out.append((np.float16(a - np.float16(1152)), np.float16(b - np.float16(1152))))
    return out


def emulate(t_, q, s, x, rows, nb):
    """Replay the consumer warps: returns y[rows][B] in float64."""
    B = x.shape[0]
    ntiles = (rows + 15) // 16
    # activations: hi/lo binary16 in fragment order, [block][seq][c] -> 8 hi then 8 lo
    xh = x.astype(np.float16)
    xl = (x - xh.astype(np.float32)).astype(np.float16)
    y = np.zeros((ntiles * 16, B))
    for t in range(ntiles):
        for b in range(nb):
            chunk = q[(t * nb + b) * QB[t_]:(t * nb + b + 1) * QB[t_]]
            A = np.zeros((2, 16, 16))  # [step][row][phys k]
            for lane in range(32):
                g, c = lane >> 2, lane & 3
                if t_ == gguf.Q4_0:
                    w = chunk[lane * 8:lane * 8 + 8].view("<u4")
                    ra, rb = decode_q4(int(w[0])), decode_q4(int(w[1]))
                elif t_ == gguf.Q8_0:
                    w = chunk[lane * 16:lane * 16 + 16].view("<u4")
                    ra, rb = decode_q8(int(w[0]), int(w[1])), decode_q8(int(w[2]), int(w[3]))
                else:
                    w = chunk[lane * 32:lane * 32 + 32].view("<u4")
                    ra = [h2(int(v)) for v in w[:4]]
                    rb = [h2(int(v)) for v in w[4:]]
                for step in range(2):
                    for row, regs in ((g, ra), (g + 8, rb)):
                        A[step, row, 2 * c], A[step, row, 2 * c + 1] = regs[2 * step]
                        A[step, row, 2 * c + 8], A[step, row, 2 * c + 9] = regs[2 * step + 1]
            D = np.zeros((16, B))
            for step in range(2):
                Bm = np.zeros((16, B))
                for n in range(B):
                    for c in range(4):
                        e = b * 32 + 8 * c
                        for part in (xh, xl):
                            frag = np.zeros(8)
                            for k in range(8):
                                frag[frag_pos(k)] = part[n, e + k]
                            pair = frag[4 * step:4 * step + 4]  # two half2 registers of this step
                            Bm[2 * c, n] += pair[0]
                            Bm[2 * c + 1, n] += pair[1]
                            Bm[2 * c + 8, n] += pair[2]
                            Bm[2 * c + 9, n] += pair[3]
                D += A[step] @ Bm
            if t_ == gguf.F16:
                y[t * 16:(t + 1) * 16] += D
            else:
                for rr in range(16):
                    so = scale_offset(nb, t * 16 + rr, b)
                    d = s[so:so + 2].view("<f2")[0]
                    y[t * 16 + rr] += float(d) * D[rr]
    return y[:rows]


@pytest.mark.parametrize("t_", [gguf.Q4_0, gguf.Q8_0, gguf.F16])
def test_offsets_are_a_bijection(t_):
    rows, nb = 32, 3
    seen = set()
    for r in range(rows):
        for i in range(nb * 32):
            off = elem_offset(t_, nb, r, i)
            span = range(off, off + 2) if t_ == gguf.F16 else [off] if t_ == gguf.Q8_0 else [(off, i & 1)]
            for v in span:
                assert v not in seen
                seen.add(v)


@pytest.mark.parametrize("t_", [gguf.Q4_0, gguf.Q8_0, gguf.F16])
@pytest.mark.parametrize("B", [1, 3])
def test_fragment_emulation_matches_dense(t_, B):
    rows, nb = 20, 2  # a partial second row tile
    rng = np.random.default_rng(t_ * 10 + B)
    w = rng.standard_normal(rows * nb * 32, dtype=np.float32) * np.float32(0.05)
    raw = np.frombuffer(synth.encode(w, t_), dtype=np.uint8)
    q, s = repack(t_, raw, rows, nb)
    x = rng.standard_normal((B, nb * 32), dtype=np.float32)
    y = emulate(t_, q, s, x, rows, nb)
    wd = O.dequant(t_, raw, rows * nb * 32).reshape(rows, nb * 32).astype(np.float64)
    ref = wd @ x.astype(np.float64).T
    assert np.allclose(y, ref, rtol=0, atol=1e-6 * np.abs(wd).sum(axis=1, keepdims=True).max())


def dp_byte_of(t_, k):
    """Byte (0..7) of element k of an 8-column group in a lane's two quant words."""
    return (k & 1) * 4 + (k >> 1) if t_ == gguf.Q4_0 else frag_pos(k)


def digits(x):
    """One 32-column block of the integer variant's records (dp_group_digits): the block exponent
    ex from the largest magnitude's float bits (mx in [2^(ex-1), 2^ex)), xi = rint(x * 2^(20-ex))
    by one exact multiply (|xi| <= 2^20), balanced base-128 digits, and the scale 2^(ex-20);
    blocks whose largest magnitude is below 2^-100 are zeros."""
    x = x.astype(np.float32)
    mx = np.float32(np.abs(x).max())
    eb = (int(mx.view(np.uint32)) >> 23) & 0xFF
    ex = eb - 126
    ok = eb != 0xFF and ex > -100
    sc = np.float32(np.ldexp(np.float32(1.0), 20 - ex)) if ok else np.float32(0.0)
    xi = np.rint(x * sc).astype(np.int64) if ok else np.zeros(32, np.int64)
    if ok:  # the multiply equals ldexp: the same integers as rintf(ldexpf(x, 20 - ex))
        assert np.array_equal(xi, np.rint(np.ldexp(x, 20 - ex)).astype(np.int64))
    p2 = ((xi + 64) & 127) - 64
    t1 = (xi - p2) >> 7
    p1 = ((t1 + 64) & 127) - 64
    p0 = (t1 - p1) >> 7
    assert np.all(np.abs(np.stack([p0, p1, p2])) <= 64)
    assert np.array_equal(p0 * 16384 + p1 * 128 + p2, xi)
    return xi, (p0, p1, p2), np.float32(np.ldexp(1.0, ex - 20)) if ok else np.float32(0.0)


def block_record(t_, x):
    """The 128-byte record of one block (kDpRecBytes layout): at d*32 + c*8 the two words of digit
    d over group c in the quants' byte order, at 96 the int -8 * sum xi (Q4_0) and 2^-s."""
    xi, pcs, sinv = digits(x)
    rec = np.zeros(128, np.uint8)
    for d in range(3):
        for c in range(4):
            for k in range(8):
                rec[d * 32 + c * 8 + dp_byte_of(t_, k)] = np.uint8(np.int64(pcs[d][8 * c + k]) & 0xFF)
    rec[96:100] = np.array([-8 * int(xi.sum()) if t_ == gguf.Q4_0 else 0], "<i4").view(np.uint8)
    rec[100:104] = np.array([sinv], "<f4").view(np.uint8)
    return rec


def imma16832(a_frag, b_frag, signed_a):
    """mma.m16n8k32 (int8): a_frag[lane] = 4 words (a0..a3), b_frag[lane] = 2 words (b0, b1) as in
    the PTX fragment layout; returns the int32 D fragments [lane][4]."""
    def bytes_of(wd, signed):
        v = np.array([(wd >> (8 * i)) & 0xFF for i in range(4)], np.int64)
        return np.where(v > 127, v - 256, v) if signed else v
    A = np.zeros((16, 32), np.int64)
    Bm = np.zeros((32, 8), np.int64)
    for lane in range(32):
        g, c = lane >> 2, lane & 3
        a0, a1, a2, a3 = a_frag[lane]
        A[g, 4 * c:4 * c + 4] = bytes_of(a0, signed_a)
        A[g + 8, 4 * c:4 * c + 4] = bytes_of(a1, signed_a)
        A[g, 16 + 4 * c:16 + 4 * c + 4] = bytes_of(a2, signed_a)
        A[g + 8, 16 + 4 * c:16 + 4 * c + 4] = bytes_of(a3, signed_a)
        b0, b1 = b_frag[lane]
        Bm[4 * c:4 * c + 4, g] = bytes_of(b0, True)
        Bm[16 + 4 * c:16 + 4 * c + 4, g] = bytes_of(b1, True)
    D = A @ Bm
    return [[D[l >> 2, 2 * (l & 3)], D[l >> 2, 2 * (l & 3) + 1], D[(l >> 2) + 8, 2 * (l & 3)],
             D[(l >> 2) + 8, 2 * (l & 3) + 1]] for l in range(32)]


def emulate_integer(t_, q, s, x, rows, nb):
    """Replay the one-sequence integer variant (mv_streamk.cuh, NT = 0) on the fragment layout:
    per tile-block the lanes' A fragments from the quant words, the B fragments from the block
    record (lane 4g + c: digit g mod 3 of group c), one mma.m16n8k32, and the lane constants that
    combine the digit columns (tile_block_dp, dp_lane); the row's four lanes are added at the end."""
    ntiles = (rows + 15) // 16
    y = np.zeros(ntiles * 16)
    u32 = lambda buf, off: int(np.frombuffer(buf[off:off + 4].tobytes(), "<u4")[0])
    for t in range(ntiles):
        acc = np.zeros((32, 2))
        for b in range(nb):
            rec = block_record(t_, x[b * 32:(b + 1) * 32])
            chunk = q[(t * nb + b) * QB[t_]:(t * nb + b + 1) * QB[t_]]
            a_frag, b_frag = [], []
            for lane in range(32):
                g, c = lane >> 2, lane & 3
                if t_ == gguf.Q4_0:
                    wx, wy = u32(chunk, lane * 8), u32(chunk, lane * 8 + 4)
                    m = 0x0F0F0F0F
                    a_frag.append((wx & m, wy & m, (wx >> 4) & m, (wy >> 4) & m))
                else:
                    wx, wy, wz, ww = (u32(chunk, lane * 16 + 4 * i) for i in range(4))
                    a_frag.append((wx, wz, wy, ww))
                boff = (g % 3) * 32 + c * 8
                b_frag.append((u32(rec, boff), u32(rec, boff + 4)))
            r = imma16832(a_frag, b_frag, signed_a=(t_ != gguf.Q4_0))
            x8 = int(np.frombuffer(rec[96:100].tobytes(), "<i4")[0])
            sinv = float(np.frombuffer(rec[100:104].tobytes(), "<f4")[0])
            for lane in range(32):
                g, c = lane >> 2, lane & 3
                ka, kb, kx = (16384, 128, 0) if c == 0 else (1, 0, 1) if c == 1 else (0, 0, 0)
                for h, row in ((0, g), (1, g + 8)):
                    v = r[lane][2 * h] * ka + r[lane][2 * h + 1] * kb + x8 * kx
                    assert abs(v) < 2 ** 30
                    d = float(s[scale_offset(nb, t * 16 + row, b):][:2].view("<f2")[0])
                    acc[lane, h] += float(v) * d * sinv
        for lane in range(32):
            g = lane >> 2
            y[t * 16 + g] += acc[lane, 0]
            y[t * 16 + g + 8] += acc[lane, 1]
    return y[:rows]


@pytest.mark.parametrize("t_", [gguf.Q4_0, gguf.Q8_0])
def test_integer_variant_emulation_matches_dense(t_):
    rows, nb = 20, 3
    rng = np.random.default_rng(7 + t_)
    w = rng.standard_normal(rows * nb * 32, dtype=np.float32) * np.float32(0.05)
    raw = np.frombuffer(synth.encode(w, t_), dtype=np.uint8)
    q, s = repack(t_, raw, rows, nb)
    x = rng.standard_normal(nb * 32).astype(np.float32) * np.float32(3.0)
    x[5] = np.float32(40.0)  # a large entry in one block
    x[64:96] = 0.0  # an all-zero block
    x[70] = np.float32(1e-35)  # a block below 2^-100: written as zeros
    y = emulate_integer(t_, q, s, x, rows, nb)
    wd = O.dequant(t_, raw, rows * nb * 32).reshape(rows, nb * 32).astype(np.float64)
    ref = wd @ x.astype(np.float64)
    # the products are exact in int32; the only rounding is of x, to half a step 2^(ex-21) of its
    # block (nothing for the blocks written as zeros, whose entries are below 2^-100), plus FP32 sums
    bound = 1e-6 * (np.abs(wd) @ np.abs(x))
    for b in range(nb):
        mx = np.abs(x[b * 32:(b + 1) * 32]).max()
        half_step = np.ldexp(1.0, int(np.frexp(mx)[1]) - 21) if mx >= 2.0 ** -100 else 2.0 ** -100
        bound += half_step * np.abs(wd[:, b * 32:(b + 1) * 32]).sum(axis=1)
    assert np.all(np.abs(y - ref) <= bound)
