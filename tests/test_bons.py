"""The BONS image reader (trixium_b200.bons) on an image the reference's own generator and writer
made (model/tinygen.py, model/bons.py:342-461): header, table, the row packets of every matvec
tensor reassembled from the channel shards, and (on a GPU) the engine matvec of each loaded
tensor against the reference's."""
import gzip
import hashlib
import os
import shutil

import numpy as np
import pytest
import torch

from oracle import ref
from trixium_b200 import bons, layout as L

from conftest import GOLDEN, load

MATVEC_KINDS = (L.KIND_TERNARY, L.KIND_TERNARY5, L.KIND_Q8)


@pytest.fixture(scope="module")
def image(tmp_path_factory):
    p = tmp_path_factory.mktemp("bons") / "tiny.img"
    with gzip.open(os.path.join(GOLDEN, "bons_tiny_l1_t5_n2.img.gz"), "rb") as src, open(p, "wb") as dst:
        shutil.copyfileobj(src, dst)
    return bons.BONSImage(str(p)), load(os.path.join(GOLDEN, "bons_tiny_l1_t5_n2.npz"))


def test_header_and_table(image):
    img, d = image
    for k in ("n_layer", "n_embd", "n_head", "n_kv_head", "head_dim", "ffn_dim", "vocab", "n_channels",
              "n_tensors", "payload_beats"):
        assert img.header[k] == int(d[k]), k
    assert [e["name"] for e in img.entries] == list(d["names"])


def test_row_packets_decode_like_the_reference_reader(image):
    img, d = image
    n = 0
    for i, e in enumerate(img.entries):
        if e["kind"] not in MATVEC_KINDS:
            continue
        pk = img.row_packets(e)
        if e["kind"] == L.KIND_Q8:
            s, v = ref.q8_decode_packed(pk, e["rows"], e["cols"])
        else:
            s, v = ref.decode_packed(pk, e["rows"], e["cols"], e["kind"])
        h = hashlib.sha256(np.ascontiguousarray(s).tobytes() + v.astype(np.int16).tobytes()).hexdigest()
        assert h == str(d[f"e{i}_sha"]), e["name"]
        n += 1
    assert n == sum(1 for k in d if k.endswith("_sha"))


def test_corrupt_payload_fails_the_crc(image, tmp_path):
    img, _ = image
    e = next(e for e in img.entries if e["kind"] == L.KIND_TERNARY5)
    raw = bytearray(np.asarray(img.data).tobytes())
    off = img.header["payload_offset"] + e["chan_base_beats"] * L.BEAT_BYTES + 40
    raw[off] ^= 0x01
    p = tmp_path / "bad.img"
    p.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="CRC"):
        bons.BONSImage(str(p)).tensor_bytes(e)


def test_not_a_bons_image(tmp_path):
    p = tmp_path / "zero.img"
    p.write_bytes(bytes(8192))
    with pytest.raises(ValueError):
        bons.BONSImage(str(p))


@pytest.mark.gpu
def test_loaded_tensors_run_on_the_engine(image):
    """Every matvec tensor of the image, loaded onto the device, gives the reference's engine
    result (model/bitexact.py matvec_ternary / matvec_q8) bit for bit."""
    from trixium_b200 import ops
    img, d = image
    ctx = ops.default_context()
    for i, e in enumerate(img.entries):
        if e["kind"] not in MATVEC_KINDS:
            continue
        dt = img.device_tensor(e)
        x8 = torch.from_numpy(d[f"e{i}_x8"]).cuda()
        y = (ops.matvec_q8 if e["kind"] == L.KIND_Q8 else ops.matvec_i8)(ctx, dt, x8).cpu().numpy()
        ctx.raise_on_error()
        assert np.array_equal(y, d[f"e{i}_y"]), e["name"]
