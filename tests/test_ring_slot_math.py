"""The ring kernels' slot arithmetic: (pos - 1) mod RING by a multiply-high with a host-computed reciprocal.

launch_ring_attn (csrc/ring_attn.cu, ring_reciprocal) sets magic = ceil(2^(63 + l) / RING) and shift = l - 1 with
l = ceil(log2 RING); ring_pm1_mod then takes z = pos - 1 (pos >= 1) or z = -pos (pos <= 0), q = umulhi64(z, magic) >> shift,
r = z - q * RING, and returns r, or RING - 1 - r for pos <= 0. This test restates those integer steps with Python
integers held to 64 bits and checks them against Python's exact modulo for every ring size the C ABI accepts
(2 .. 128) over positions at the edges of the int64 range, around multiples of the ring, and at random."""
import random

INT64_MIN, INT64_MAX = -(1 << 63), (1 << 63) - 1
MASK64 = (1 << 64) - 1


def reciprocal(d):
    """ring_reciprocal: magic and shift for 2 <= d <= 128."""
    l = 1
    while (1 << l) < d:
        l += 1
    magic = ((1 << (63 + l)) + d - 1) // d
    assert magic <= MASK64
    return magic, l - 1


def pm1_mod(pos, d, magic, shift):
    """ring_pm1_mod, step by step in 64-bit unsigned arithmetic."""
    up = pos & MASK64
    ge1 = pos >= 1
    z = (up - 1) & MASK64 if ge1 else (0 - up) & MASK64
    q = ((z * magic) >> 64) >> shift                        # __umul64hi, then the shift
    r = (z - q * d) & MASK64
    assert 0 <= r < d, (pos, d, r)
    return r if ge1 else d - 1 - r


def positions(d, rng):
    edge = [0, 1, 2, d - 1, d, d + 1, 2 * d - 1, 2 * d, 2**31 - 1, 2**31, 2**32 - 1, 2**32, 2**32 + 1,
            2**62, 2**63 - 64, INT64_MAX, INT64_MAX - 1, -1, -2, -d, -d - 1, INT64_MIN, INT64_MIN + 1]
    near = [k * d + o for k in (1, 7, 2**20, 2**40 // d, INT64_MAX // d) for o in (-1, 0, 1)]
    rand = [rng.randrange(INT64_MIN, INT64_MAX + 1) for _ in range(300)] + [rng.randrange(0, 2**40) for _ in range(300)]
    return [p for p in edge + near + rand if INT64_MIN <= p <= INT64_MAX]


def test_slot_arithmetic_is_exact_for_every_ring_size():
    rng = random.Random(1234)
    for d in range(2, 129):
        magic, shift = reciprocal(d)
        for pos in positions(d, rng):
            assert pm1_mod(pos, d, magic, shift) == (pos - 1) % d, (pos, d)


def test_write_slot_follows_from_the_newest_slot():
    # ring_slot_after(pm1, f, RING) = (pm1 + 1 + f) % RING is the slot of frame pos + f
    rng = random.Random(99)
    for d in (2, 3, 17, 72, 88, 128):
        magic, shift = reciprocal(d)
        for pos in positions(d, rng)[:200]:
            pm1 = pm1_mod(pos, d, magic, shift)
            for f in range(18):
                if pos + f <= INT64_MAX:
                    assert (pm1 + 1 + f) % d == (pos + f) % d
