"""Routed experts read from safetensors shards (k3c_ckpt_*, k3c_expert_ref / _read) against
the reference's own shard index and expert loader (k3_st_open, k3_expert_ref,
k3_expert_load_direct compiled into oracle/_ref) and against the bytes the test wrote."""
import ctypes as C
import json
import os

import numpy as np
import pytest

import ckpt_util as ck
from ckpt_util import EXPERT, build_checkpoint, write_raw, write_shard

REF = pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).ref_available()")


@pytest.fixture(scope="module")
def ckpt_dir(tmp_path_factory, k3):
    d = str(tmp_path_factory.mktemp("ckpt"))
    want = build_checkpoint(d, k3.synth.rng(2026))
    return d, want


def test_index_and_find(k3, ckpt_dir):
    d, _ = ckpt_dir
    ck = k3.Checkpoint(d)
    assert ck.shards == 2
    t = ck.find("model.norm_bf16")
    assert (t.shard, t.dtype, t.ndim, t.shape[0], t.nbytes) == (0, 2, 1, 7, 14)   # K3C_DT_BF16
    t = ck.find(EXPERT.format(2, 0, "w2", "weight_scale"))
    assert t.shard == 1 and t.ndim == 2 and (t.shape[0], t.shape[1]) == (256, 4)
    with pytest.raises(k3.K3CError):
        ck.find("model.absent")
    ck.close()


def test_expert_runs_match_written_bytes(k3, ckpt_dir):
    d, want = ckpt_dir
    ck = k3.Checkpoint(d)
    for (layer, expert), (canon, _) in want.items():
        r = ck.expert_ref(layer, expert)
        payload = ck.read_expert(r)
        # assemble the canonical order from the run's own offsets
        got = b"".join(payload[r.m[i].p_off:r.m[i].p_off + r.m[i].p_bytes].tobytes() +
                       payload[r.m[i].s_off:r.m[i].s_off + r.m[i].s_bytes].tobytes() for i in range(3))
        assert got == canon
        assert r.nbytes == len(canon)
    assert ck.expert_ref(1, 0).contiguous == 1 and ck.expert_ref(1, 1).contiguous == 1
    assert ck.expert_ref(1, 2).contiguous == 0
    assert ck.expert_ref(1, 1).m[2].p_off == 0          # w3 first in the file
    with pytest.raises(k3.K3CError, match="spans shards"):
        ck.expert_ref(1, 3)
    with pytest.raises(k3.K3CError, match="missing"):
        ck.expert_ref(1, 9)


@REF
def test_expert_runs_match_reference_loader(k3, ora, ckpt_dir):
    d, want = ckpt_dir
    ck = k3.Checkpoint(d)
    for layer, expert in list(want) + [(1, 3), (1, 9)]:
        st, rr, rb = ora.ref_expert_read(d, layer, expert, k3.ExpertRunC, 1 << 20)
        try:
            r = ck.expert_ref(layer, expert)
        except k3.K3CError:
            assert st == -2, (layer, expert)
            continue
        assert st == r.nbytes
        assert bytes(r) == bytes(rr)                    # every field of K3ExpertRef
        assert ck.read_expert(r).tobytes() == rb.tobytes()


def _bad(d, name, tensors, hdr_len=None, **kw):
    os.makedirs(d, exist_ok=True)
    p = os.path.join(d, name)
    write_shard(p, tensors, **kw)
    if hdr_len is not None:
        with open(p, "r+b") as f:
            f.write(int(hdr_len).to_bytes(8, "little"))
    return d


@pytest.mark.parametrize("case", ["hdr_len", "span", "eof", "dtype", "dup"])
def test_malformed_shards_are_rejected(k3, ora, tmp_path, case):
    d = str(tmp_path / case)
    a = np.arange(16, dtype=np.uint8)
    if case == "hdr_len":
        _bad(d, "m.safetensors", [("x", a, None)], hdr_len=1 << 40)
    elif case == "span":       # shape says 4 bytes, the offsets 16
        _bad(d, "m.safetensors", [("x", a, None)])
        p = os.path.join(d, "m.safetensors")
        raw = open(p, "rb").read().replace(b'"shape": [16]', b'"shape": [4] ')
        open(p, "wb").write(raw)
    elif case == "eof":
        _bad(d, "m.safetensors", [("x", a, None)])
        p = os.path.join(d, "m.safetensors")
        raw = open(p, "rb").read()
        open(p, "wb").write(raw[:-3])
    elif case == "dtype":
        _bad(d, "m.safetensors", [("x", a.view(np.uint64), "F64")])
    else:                      # the same name in two shards
        _bad(d, "a.safetensors", [("x", a, None)])
        _bad(d, "b.safetensors", [("x", a, None)])
    with pytest.raises(k3.K3CError):
        k3.Checkpoint(d)
    if ora.ref_available():
        st, _, _ = ora.ref_expert_read(d, 0, 0, k3.ExpertRunC, 4096)
        assert st == -1


def test_unaligned_buffer_reads_buffered(k3, ckpt_dir):
    """A destination that is not page aligned cannot take an O_DIRECT read: the run is read
    through the page cache into the buffer's start instead."""
    d, want = ckpt_dir
    ck = k3.Checkpoint(d)
    r = ck.expert_ref(1, 0)
    aligned = k3.aligned_host_buffer(r.nbytes + 2 * 4096 + 64)
    buf = aligned[8:]                                    # 8 bytes past a page boundary
    po = C.c_int64(-1)
    n = k3.lib().k3c_expert_read(ck.h, C.byref(r), C.c_void_p(buf.ctypes.data), buf.size, C.byref(po))
    assert n == r.nbytes and po.value == 0
    assert buf[:n].tobytes() == ck.read_expert(r).tobytes()


QUIRKS = (
    '{ "__metadata__" : {"a": [1, 2.5e3, {"b": "x\\"y]}"}], "n": null, "t": true},\n'
    ' "we\\"ird\\\\name\\/u\\u0041\\u00e9" : {"dtype":"U8","shape":[3],"data_offsets":[0,3]},\n'
    '\t"scalar": {"shape": [], "dtype": "F32", "data_offsets": [3, 7]},'
    ' "empty": {"dtype": "BF16", "shape": [0, 5], "data_offsets": [7, 7]},'
    ' "extra": {"dtype":"U8","shape":[2,2],"data_offsets":[7,11], "other": {"k": [1, "]"]}}, }'
)
QUIRK_NAMES = ['we"ird\\name/uA?', "scalar", "empty", "extra", "missing"]


def test_header_quirks_match_reference_index(k3, ora, tmp_path):
    """Escapes in names (a non-ASCII code point reads as '?'), nested metadata holding
    brackets inside strings, tabs and newlines, a scalar, a zero-size tensor, an unknown key
    holding an object, a trailing comma: every name resolves as in the reference's index."""
    d = str(tmp_path)
    write_raw(f"{d}/m.safetensors", QUIRKS, bytes(range(11)))
    ck = k3.Checkpoint(d)
    got = []
    for n in QUIRK_NAMES:
        try:
            t = ck.find(n)
            got.append((1, t.shard, t.dtype, t.ndim, t.off, t.nbytes,
                        t.shape[0] if t.ndim > 0 else 0, t.shape[1] if t.ndim > 1 else 0))
        except k3.K3CError:
            got.append((0,) * 8)
    assert got[0][0] == 1 and got[1][3] == 0 and got[2][5] == 0 and got[4][0] == 0
    if ora.ref_available():
        assert got == ora.ref_st_find(d, QUIRK_NAMES)


@pytest.mark.parametrize("hdr", [
    '{"x": {"dtype": "U8", "shape": [1, 1, 1, 1, 1], "data_offsets": [0, 1]}}',   # rank 5
    '{"x": {"dtype": "U8", "shape": [1], "data_offsets": [0, 1]}, "x": {"dtype": "U8", "shape": [1], "data_offsets": [1, 2]}}',
    '{"x": {"dtype": "U8", "shape": [2]}}',                                       # no offsets
    '["x"]',                                                                      # not an object
])
def test_bad_headers_rejected_like_reference(k3, ora, tmp_path, hdr):
    d = str(tmp_path)
    write_raw(f"{d}/m.safetensors", hdr, b"\0\0")
    with pytest.raises(k3.K3CError):
        k3.Checkpoint(d)
    if ora.ref_available():
        assert ora.ref_st_find(d, ["x"]) is None


# ------------------------------------------------------------------ packed (draft) trunk
REF_INT8_TRUNK = "/root/reference/tools/int8_trunk.py"


def _trunk_layers(seed):
    g = np.random.default_rng(seed)

    def bf(r, c):
        return ck.bf16_bits_np(g.standard_normal((r, c), dtype=np.float32) * np.float32(0.05))

    layers = []
    for li in range(2):
        p = f"language_model.model.layers.{li}."
        down = bf(64, 96) if li == 0 else np.zeros((64, 96), np.uint16)   # an all-zero matrix: scale 1
        layers.append([(p + "block_sparse_moe.down_proj.weight", down),
                       (p + "block_sparse_moe.up_proj.weight", bf(96, 64)),
                       (p + "block_sparse_moe.shared_experts.w1.weight", bf(32, 96)),
                       (p + "post_attention_layernorm.weight", np.ones(96, np.float32)),
                       (p + "block_sparse_moe.gate.e_score_correction_bias", g.standard_normal(8, dtype=np.float32))])
    return layers


def test_int8_trunk_restatement_matches_reference_tool(tmp_path):
    """tests/ckpt_util.int8_trunk (the draft trunk the layer tests read) writes the same bytes and
    manifest as the reference's own tools/int8_trunk.py on the same bf16 packed trunk, including
    an all-zero matrix (scale 1)."""
    import os
    import subprocess
    import sys
    if not os.path.exists(REF_INT8_TRUNK):
        pytest.skip("the reference tree is not present")
    src = str(tmp_path / "bf16")
    ck.write_bf16_trunk(src, _trunk_layers(1))
    ck.int8_trunk(src, str(tmp_path / "ours"))
    subprocess.run([sys.executable, REF_INT8_TRUNK, src, str(tmp_path / "ref")], check=True, capture_output=True)
    assert open(tmp_path / "ours" / "trunk.bin", "rb").read() == open(tmp_path / "ref" / "trunk.bin", "rb").read()
    assert json.load(open(tmp_path / "ours" / "trunk.json")) == json.load(open(tmp_path / "ref" / "trunk.json"))


def test_trunk_reader_knows_i8r(k3, tmp_path):
    """k3c_trunk_*: every tensor of a draft trunk by (layer, name) with its dtype (I8R for the
    quantised matrices, F32 for the rest), absolute offset and shape; the bytes read (O_DIRECT
    into an aligned buffer, buffered otherwise) are the file's."""
    src, out = str(tmp_path / "bf16"), str(tmp_path / "i8")
    ck.write_bf16_trunk(src, _trunk_layers(2))
    man = ck.int8_trunk(src, out)
    raw = open(tmp_path / "i8" / "trunk.bin", "rb").read()
    tr = k3.Trunk(out)
    assert tr.layers == 2
    for li, lay in enumerate(man["layers"]):
        for name, t in lay["tensors"].items():
            got = tr.find(li, name)
            assert got.dtype == (k3.DT_I8R if t["dtype"] == "I8R" else {"F32": 4, "BF16": 2}[t["dtype"]])
            assert got.off == lay["file_off"] + t["off"] and got.nbytes == t["nbytes"]
            assert [got.shape[i] for i in range(got.ndim)] == t["shape"]
            assert tr.read(got).tobytes() == raw[got.off:got.off + got.nbytes]
    rows = tr.read(tr.find(0, "language_model.model.layers.0.block_sparse_moe.down_proj.weight")).reshape(64, 100)
    assert np.all(rows[:, :4].view(np.float32) > 0)
    with pytest.raises(k3.K3CError, match="not in layer"):
        tr.find(1, "nope")
    tr.close()


@pytest.mark.parametrize("edit,match", [
    (lambda t: t.update(nbytes=t["nbytes"] - 1), "spans"),
    (lambda t: t.update(dtype="Q4"), "unsupported dtype"),
    (lambda t: t.update(off=10 ** 9), "runs past"),
    (lambda t: t.update(shape=[64]), "not 2-D"),
])
def test_trunk_reader_refuses_bad_manifests(k3, tmp_path, edit, match):
    src, out = str(tmp_path / "bf16"), str(tmp_path / "i8")
    ck.write_bf16_trunk(src, _trunk_layers(3))
    man = ck.int8_trunk(src, out)
    edit(man["layers"][0]["tensors"]["language_model.model.layers.0.block_sparse_moe.down_proj.weight"])
    json.dump(man, open(tmp_path / "i8" / "trunk.json", "w"))
    with pytest.raises(k3.K3CError, match=match):
        k3.Trunk(out)
