"""Reader of BONS weight images: the header, the tensor table, and a tensor's row packets
reassembled from its channel shards onto the device.

The file contract is the reference converter's (model/layout.py:226-333; reader
model/bons.py:476-525): a 4 KiB header, a table of 64-byte entries padded to 4 KiB, then one
payload per engine channel, all of `payload_beats` 32-byte beats.  A row-sharded tensor keeps
rows [c*M/N, (c+1)*M/N) in channel c at the same relative beat offset in every channel, so the
tensor's row packets are the channels' slices in channel order; a replicated tensor
(FLAG_REPLICATED) is read from channel 0.  The struct layouts below are the file format and so
follow the reference's field for field.
"""

import struct
import zlib

import numpy as np

from . import layout as L

MAGIC = 0x534E4F42                      # "BONS"
VERSIONS = (2, 3)
HEADER_SIZE = 4096
ENTRY_SIZE = 64
FLAG_REPLICATED = 0x01
FLAG_KSEG = 0x02

# Tensor roles (model/layout.py:99-121).
(ROLE_TOK_EMB, ROLE_OUT_NORM, ROLE_LM_HEAD, ROLE_ATTN_NORM, ROLE_ATTN_Q, ROLE_ATTN_K, ROLE_ATTN_V, ROLE_ATTN_OUT,
 ROLE_ATTN_Q_NORM, ROLE_ATTN_K_NORM, ROLE_FFN_NORM, ROLE_FFN_GATE, ROLE_FFN_UP, ROLE_FFN_DOWN, ROLE_ROPE_TAB,
 ROLE_TOK_EMB16, ROLE_TOK_EMB16_EXP) = range(17)
(ROLE_ATTN_QKV, ROLE_ATTN_ZGATE, ROLE_SSM_OUT, ROLE_SSM_BETA, ROLE_SSM_ALPHA, ROLE_SSM_CONV, ROLE_SSM_A, ROLE_SSM_DT,
 ROLE_SSM_NORM, ROLE_HADAMARD) = range(17, 27)


def hadamard_layer(width_index, block_index):
    """The entry `layer` of a rotation block tensor: width index * 256 + block (model/layout.py:124-128)."""
    return width_index * 256 + block_index

# Header (little-endian), model/layout.py:242-257: the fixed fields at 0..111 ...
_HEADER = struct.Struct("<IIIIIIIIIIfIIIIIQII32s")
_HEADER_KEYS = ("magic", "version", "n_layer", "n_embd", "n_head", "n_kv_head", "head_dim", "ffn_dim",
                "vocab", "rope_theta", "rms_eps", "max_ctx", "n_channels", "n_tensors", "table_offset",
                "payload_offset", "payload_beats", "mode", "table_crc32", "tokenizer_sha256")
# ... and the hybrid fields of v3 at 112 (all zero for a plain Qwen3 model).
_HEADER_V3 = struct.Struct("<QQHHHHHHHBBIIII")
_HEADER_V3_OFF = 112
# Tensor table entry, model/layout.py:318-322.
_ENTRY = struct.Struct("<BBBBHHIIQQIBB2x24s")
_ENTRY_KEYS = ("role", "kind", "flags", "kseg", "layer", "group", "rows", "cols", "chan_base_beats",
               "chan_len_beats", "crc32", "bias", "rshift", "name")


def parse_header(buf):
    h = dict(zip(_HEADER_KEYS, _HEADER.unpack_from(buf, 0)))
    if h["magic"] != MAGIC:
        raise ValueError("not a BONS image")
    if h["version"] not in VERSIONS:
        raise ValueError(f"BONS version {h['version']} is not one of {VERSIONS}")
    v3 = _HEADER_V3.unpack_from(buf, _HEADER_V3_OFF) if h["version"] >= 3 else (0,) * 15
    lt = v3[0] | (v3[1] << 64)
    h["layer_types"] = tuple("deltanet" if (lt >> l) & 1 else "attn" for l in range(h["n_layer"]))
    (h["dn_num_v_heads"], h["dn_num_k_heads"], h["dn_k_head_dim"], h["dn_v_head_dim"], h["dn_conv_kernel"],
     h["rope_dims"], h["hadamard_block"], h["attn_gated"], h["hyb_flags"]) = v3[2:11]
    h["hadamard_widths"] = tuple(w for w in v3[11:15] if w)
    return h


def parse_entry(buf, off):
    e = dict(zip(_ENTRY_KEYS, _ENTRY.unpack_from(buf, off)))
    e["name"] = e["name"].rstrip(b"\x00").decode(errors="replace")
    return e


class BONSImage:
    """A BONS image on the host (memory-mapped).  `entries` keeps the table order; `find` looks a
    tensor up by name, or by (role, layer) where 24-byte names collide."""

    def __init__(self, path):
        self.data = np.memmap(path, dtype=np.uint8, mode="r")
        if self.data.size < HEADER_SIZE:
            raise ValueError("not a BONS image: shorter than its header")
        self.header = parse_header(bytes(self.data[:HEADER_SIZE]))
        h = self.header
        t0, n = h["table_offset"], h["n_tensors"]
        table = bytes(self.data[t0:t0 + n * ENTRY_SIZE])
        if len(table) != n * ENTRY_SIZE:
            raise ValueError("truncated tensor table")
        if zlib.crc32(table) & 0xFFFFFFFF != h["table_crc32"]:
            raise ValueError("tensor table CRC mismatch")
        self.entries = [parse_entry(table, i * ENTRY_SIZE) for i in range(n)]
        end = h["payload_offset"] + h["n_channels"] * h["payload_beats"] * L.BEAT_BYTES
        if self.data.size < end:
            raise ValueError("truncated payload")

    def find(self, name=None, role=None, layer=None):
        for e in self.entries:
            if (name is None or e["name"] == name) and (role is None or e["role"] == role) and \
                    (layer is None or e["layer"] == layer):
                return e
        raise KeyError(name if name is not None else (role, layer))

    def channel_slice(self, e, channel):
        """The entry's bytes in one channel's payload."""
        h = self.header
        start = h["payload_offset"] + (channel * h["payload_beats"] + e["chan_base_beats"]) * L.BEAT_BYTES
        return self.data[start:start + e["chan_len_beats"] * L.BEAT_BYTES]

    def tensor_bytes(self, e, check_crc=True):
        """The tensor's bytes: its row packets in row order (every channel's shard in turn), or
        channel 0's copy of a replicated tensor.  The entry's CRC32 covers the payload channel by
        channel (model/bons.py write_image)."""
        chans = 1 if e["flags"] & FLAG_REPLICATED else self.header["n_channels"]
        out = np.concatenate([np.asarray(self.channel_slice(e, c)) for c in range(chans)])
        if check_crc:
            crc = 0
            for c in range(self.header["n_channels"]):
                crc = zlib.crc32(bytes(self.channel_slice(e, c)), crc)
            if crc & 0xFFFFFFFF != e["crc32"]:
                raise ValueError(f"{e['name']}: payload CRC mismatch")
        return out

    def row_packets(self, e):
        """The row packets of a matvec tensor (ternary kinds or KIND_Q8) trimmed to its rows."""
        kind, rows, cols = e["kind"], e["rows"], e["cols"]
        if kind in L.TERNARY_KINDS:
            rb = L.row_bytes(cols, kind)
        elif kind == L.KIND_Q8:
            rb = L.q8_row_bytes(cols)
        else:
            raise ValueError(f"{e['name']}: kind {kind} is not a matvec tensor")
        b = self.tensor_bytes(e)
        if b.size < rows * rb:
            raise ValueError(f"{e['name']}: {b.size} bytes hold fewer than {rows} rows of {rb}")
        return b[:rows * rb]

    def plain_rows(self, e):
        """An unscaled tensor (KIND_F32, KIND_NORM16, KIND_F16) as a (rows, cols) numpy array: each
        row's values from the start of its beat-padded row (model/bons.py:170-200)."""
        dtype = {L.KIND_F32: np.float32, L.KIND_NORM16: np.int16, L.KIND_F16: np.float16}[e["kind"]]
        rb = L.plain_row_bytes(e["cols"], e["kind"])
        b = np.asarray(self.tensor_bytes(e))
        if b.size < e["rows"] * rb:
            raise ValueError(f"{e['name']}: {b.size} bytes hold fewer than {e['rows']} rows of {rb}")
        width = np.dtype(dtype).itemsize * e["cols"]
        rows = b[:e["rows"] * rb].reshape(e["rows"], rb)[:, :width]
        return np.ascontiguousarray(rows).view(dtype).reshape(e["rows"], e["cols"])

    def entries_of(self, role, layer=0, kind=None):
        """The entries of (role, layer), optionally of one kind, in table order."""
        return [e for e in self.entries if e["role"] == role and e["layer"] == layer and
                (kind is None or e["kind"] == kind)]

    def matvec_entries(self, role, layer=0):
        """The matvec tensor of (role, layer) as its K-segments in order (FLAG_KSEG, the entries'
        kseg field; model/mirror.py:635-643), or the one entry of an unsegmented tensor."""
        es = [e for e in self.entries_of(role, layer)
              if e["kind"] in L.TERNARY_KINDS or e["kind"] == L.KIND_Q8]
        if not es:
            raise KeyError((role, layer))
        if es[0]["flags"] & FLAG_KSEG:
            return sorted([e for e in es if e["flags"] & FLAG_KSEG], key=lambda e: e["kseg"])
        return es[:1]

    def embedding_bfp16(self):
        """The int16 embedding table (ROLE_TOK_EMB16, [vocab][dim] mantissas) and its per-row
        exponents (ROLE_TOK_EMB16_EXP, 16 per beat): row t is mant[t] * 2^exp[t]
        (model/mirror.py:777-783).  None when the image has no table."""
        m = self.entries_of(ROLE_TOK_EMB16, 0, L.KIND_NORM16)
        x = self.entries_of(ROLE_TOK_EMB16_EXP, 0, L.KIND_NORM16)
        if not m or not x:
            return None
        mant = self.plain_rows(m[0])
        exps = self.plain_rows(x[0]).reshape(-1)[:mant.shape[0]].astype(np.int32)
        return mant, exps

    def device_tensor(self, e, device=None):
        """The tensor on the device as an ops.DeviceTensor carrying the entry's B and R."""
        from . import ops
        if isinstance(e, str):
            e = self.find(e)
        return ops.DeviceTensor.from_packed(np.ascontiguousarray(self.row_packets(e)), e["rows"], e["cols"],
                                            e["kind"], e["bias"], e["rshift"], device=device)
