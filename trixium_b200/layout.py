"""Row-packet geometry of a ternary tensor, as the B200 kernels read it.

A tensor of `rows` x `cols` weights (cols a multiple of the 128-weight group) is stored as one
packet per output row, packets back to back (reference contract: model/layout.py:17-30):

    [ S scale beats: G fp16 group scales, 16 per 32-byte beat, zero padded ]
    [ code bytes: 2-bit (kind 0) or 5 trits per byte (kind 5), row padded to 32 bytes ]

* kind 0 (KIND_TERNARY, model/layout.py:46): code j of a group sits in byte j//4 at bits
  2*(j%4) (model/bons.py:157-160); one group = 32 bytes.
* kind 5 (KIND_TERNARY5, model/layout.py:50, :81): a group is 26 bytes; lane 5*i+k is the
  base-3 digit k of byte i (model/bons.py:115-123); lanes 128 and 129 are zero padding; a byte
  above 242 is invalid (gateware/core/trit5.py:33-45 decodes it to code 3).

The numbers here are restated from model/layout.py:184-217 (row_groups, scale_beats,
code_beats, mem_code_beats, row_beats) and model/layout.py:219-223 (shard_rows).
"""

BEAT_BYTES = 32
GROUP = 128
GROUP_Q8 = 32
SCALES_PER_BEAT = 16
TRIT5_GROUP_BYTES = 26

KIND_TERNARY = 0      # 2-bit codes
KIND_Q8 = 1
KIND_F16 = 2
KIND_F32 = 3
KIND_NORM16 = 4
KIND_TERNARY5 = 5     # 5 trits per byte

TERNARY_KINDS = (KIND_TERNARY, KIND_TERNARY5)


def ceil_div(a, b):
    return -(-a // b)


def groups(cols):
    if cols % GROUP:
        raise ValueError(f"cols {cols} is not a multiple of the {GROUP}-weight group")
    return cols // GROUP


def scale_bytes(cols):
    """Bytes of the scale region at the head of each row packet (whole beats)."""
    return ceil_div(groups(cols), SCALES_PER_BEAT) * BEAT_BYTES


def code_bytes(cols, kind):
    """Bytes of codes per row actually used (before the row's beat padding)."""
    g = groups(cols)
    if kind == KIND_TERNARY:
        return 32 * g
    if kind == KIND_TERNARY5:
        return TRIT5_GROUP_BYTES * g
    raise ValueError(f"not a ternary kind: {kind}")


def row_bytes(cols, kind):
    """Bytes of one row packet in memory (model/layout.py:215-217 times BEAT_BYTES)."""
    return scale_bytes(cols) + ceil_div(code_bytes(cols, kind), BEAT_BYTES) * BEAT_BYTES


def q8_groups(cols):
    """Groups of a KIND_Q8 row: 32 int8 weights (one beat) per fp16 scale (model/layout.py:41,47)."""
    if cols % GROUP_Q8:
        raise ValueError(f"cols {cols} is not a multiple of the {GROUP_Q8}-weight Q8 group")
    return cols // GROUP_Q8


def q8_row_bytes(cols):
    """Bytes of one KIND_Q8 row packet: ceil(G/16) scale beats, then G beats of int8 weights
    (model/layout.py:189-217 with code_beats = cols/32)."""
    g = q8_groups(cols)
    return (ceil_div(g, SCALES_PER_BEAT) + g) * BEAT_BYTES


def plain_row_bytes(cols, kind):
    """Bytes of one row of an unscaled tensor: fp32 (KIND_F32), int16 (KIND_NORM16) or fp16
    (KIND_F16) values, the row padded to whole beats (model/layout.py:189-217, no scale beats)."""
    width = {KIND_F32: 4, KIND_NORM16: 2, KIND_F16: 2}[kind]
    return ceil_div(width * cols, BEAT_BYTES) * BEAT_BYTES


def tensor_bytes(rows, cols, kind):
    return rows * row_bytes(cols, kind)


def algorithmic_bytes(rows, cols, kind):
    """Bytes a matvec must stream per row without padding: the G scales plus the G code
    groups (the roofline numerator; equals the packet bytes when there is no padding)."""
    g = groups(cols)
    per_group = (32 if kind == KIND_TERNARY else TRIT5_GROUP_BYTES) + 2
    return rows * g * per_group


def shard_rows(rows, n, k):
    """Row range [start, count) of shard k of n (block sharding, model/layout.py:219-223)."""
    if rows % n:
        raise ValueError(f"rows {rows} not divisible by {n} shards")
    per = rows // n
    return k * per, per
