"""A small safetensors writer for tests: shards laid out exactly as asked (tensor order,
filler tensors between them), so the expert loader meets contiguous, reordered, scattered and
cross-shard runs. Test infrastructure only."""
import json
import os
import struct

import numpy as np

EXPERT = "language_model.model.layers.{}.block_sparse_moe.experts.{}.{}.{}"
_DT = {np.uint8: "U8", np.float32: "F32", np.uint16: "BF16", np.float16: "F16"}


def write_shard(path, tensors, metadata=None, header_pad=0):
    """tensors: list of (name, numpy array, dtype string or None) written in list order,
    back to back. header_pad adds spaces to the JSON header (shifts every data offset)."""
    hdr, off, blobs = {}, 0, []
    if metadata is not None:
        hdr["__metadata__"] = metadata
    for name, a, dt in tensors:
        a = np.ascontiguousarray(a)
        b = a.tobytes()
        hdr[name] = {"dtype": dt or _DT[a.dtype.type], "shape": list(a.shape),
                     "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    js = json.dumps(hdr).encode() + b" " * header_pad
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(js)))
        f.write(js)
        for b in blobs:
            f.write(b)


def expert_tensors(g, layer, expert, hidden, inter, order=("w1", "w2", "w3")):
    """The six tensors of one expert (packed U8 [rows][cols/2], scales U8 [rows][cols/32]) in
    the given matrix order, and their canonical run bytes (w1.p w1.s w2.p w2.s w3.p w3.s)."""
    shapes = {"w1": (inter, hidden), "w3": (inter, hidden), "w2": (hidden, inter)}
    arrs = {}
    for w, (r, c) in shapes.items():
        arrs[w] = (g.integers(0, 256, (r, c // 2), dtype=np.uint8),
                   g.integers(118, 125, (r, c // 32), dtype=np.uint8))
    out = []
    for w in order:
        out.append((EXPERT.format(layer, expert, w, "weight_packed"), arrs[w][0], None))
        out.append((EXPERT.format(layer, expert, w, "weight_scale"), arrs[w][1], None))
    canon = b"".join(arrs[w][0].tobytes() + arrs[w][1].tobytes() for w in ("w1", "w2", "w3"))
    expert_dict = dict(gate_p=arrs["w1"][0], gate_s=arrs["w1"][1], up_p=arrs["w3"][0],
                       up_s=arrs["w3"][1], down_p=arrs["w2"][0], down_s=arrs["w2"][1])
    return out, canon, expert_dict


def build_checkpoint(d, g, hidden=256, inter=128):
    """Two shards. Layer 1 experts: 0 contiguous in canonical order after an odd-sized filler
    (an unaligned run start); 1 contiguous with its matrices in the order w3, w1, w2; 2 with a
    filler between w1 and w2 (scattered); 3 with w3 in the second shard. Layer 2 expert 0
    contiguous in the second shard. Returns {(layer, expert): (canonical bytes, expert dict)}."""
    os.makedirs(d, exist_ok=True)
    want = {}
    a, b = [], []
    a.append(("model.filler_a", g.integers(0, 256, 37, dtype=np.uint8), None))
    t, c, e = expert_tensors(g, 1, 0, hidden, inter)
    a += t
    want[(1, 0)] = (c, e)
    t, c, e = expert_tensors(g, 1, 1, hidden, inter, order=("w3", "w1", "w2"))
    a += t
    want[(1, 1)] = (c, e)
    t, c, e = expert_tensors(g, 1, 2, hidden, inter)
    a += t[:2] + [("model.filler_b", np.arange(5, dtype=np.float32), None)] + t[2:]
    want[(1, 2)] = (c, e)
    t, c, e = expert_tensors(g, 1, 3, hidden, inter)
    a += t[:4]
    b += t[4:]
    a.append(("model.norm_bf16", np.arange(7, dtype=np.uint16), "BF16"))
    t, c, e = expert_tensors(g, 2, 0, hidden, inter)
    b = [("model.filler_c", g.integers(0, 256, 4099, dtype=np.uint8), None)] + b + t
    want[(2, 0)] = (c, e)
    write_shard(os.path.join(d, "model-00001-of-00002.safetensors"), a,
                metadata={"format": "pt", "note": 'a {nested} "value", [1, 2]'}, header_pad=3)
    write_shard(os.path.join(d, "model-00002-of-00002.safetensors"), b)
    return want


def write_raw(path, header, data):
    """A shard from a header given as raw JSON text (for headers no serializer writes:
    escapes, trailing commas, odd whitespace) and its data bytes."""
    js = header.encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(js)))
        f.write(js)
        f.write(data)


# ------------------------------------------------------------------ packed trunk
TRUNK_ALIGN = 4096


def bf16_bits_np(a):
    """fp32 -> bf16 bit patterns, round to nearest even (finite values)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def write_bf16_trunk(directory, layers):
    """A packed trunk in the layout tools/pack_trunk.py writes: trunk.bin with one run per
    layer starting and ending on a 4096-byte boundary, trunk.json {"n_layers", "align",
    "layers": [{"layer", "shard", "run_start", "nbytes", "file_off", "tensors": {name: {"off",
    "nbytes", "dtype", "shape"}}}]}. layers: list of lists of (name, array) -- uint16 arrays
    are BF16 bit patterns, float32 arrays F32."""
    os.makedirs(directory, exist_ok=True)
    man = {"n_layers": len(layers), "align": TRUNK_ALIGN, "layers": []}
    with open(os.path.join(directory, "trunk.bin"), "wb") as f:
        for li, tensors in enumerate(layers):
            f.write(b"\0" * ((-f.tell()) % TRUNK_ALIGN))
            file_off, off, ts = f.tell(), 0, {}
            for name, a in tensors:
                a = np.ascontiguousarray(a)
                b = a.tobytes()
                ts[name] = {"off": off, "nbytes": len(b), "dtype": _DT[a.dtype.type], "shape": list(a.shape)}
                f.write(b)
                off += len(b)
            f.write(b"\0" * ((-f.tell()) % TRUNK_ALIGN))
            man["layers"].append({"layer": li, "shard": "model.safetensors", "run_start": 0,
                                  "nbytes": (off + TRUNK_ALIGN - 1) & ~(TRUNK_ALIGN - 1),
                                  "file_off": file_off, "tensors": dict(sorted(ts.items()))})
    with open(os.path.join(directory, "trunk.json"), "w") as f:
        json.dump(man, f)
    return man


def quant_rows_int8(f32_2d):
    """Per-row int8 rows [f32 scale][int8 * cols]: scale = max|row| / 127 in fp32 (1 for an all-zero
    row), q = round-half-even(f / scale) clipped to [-128, 127] -- tools/int8_trunk.py:33-45."""
    amax = np.abs(f32_2d).max(axis=1)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    scale[scale == 0] = np.float32(1.0)
    q = np.rint(f32_2d / scale[:, None]).clip(-128, 127).astype(np.int8)
    rows = np.empty((f32_2d.shape[0], 4 + f32_2d.shape[1]), np.uint8)
    rows[:, :4] = scale.view(np.uint8).reshape(-1, 4)
    rows[:, 4:] = q.view(np.uint8)
    return rows


def int8_trunk(src, out):
    """The draft trunk from a bf16 packed trunk, as tools/int8_trunk.py:58-98 makes it: every
    2-D BF16 tensor becomes I8R rows, everything else is copied; runs keep their order and
    4096-byte alignment, tensors are laid out in ascending source offset."""
    os.makedirs(out, exist_ok=True)
    man = json.load(open(os.path.join(src, "trunk.json")))
    raw = open(os.path.join(src, "trunk.bin"), "rb").read()
    new = {k: v for k, v in man.items() if k != "layers"}
    new["layers"] = []
    with open(os.path.join(out, "trunk.bin"), "wb") as f:
        for lay in man["layers"]:
            run = raw[lay["file_off"]:lay["file_off"] + lay["nbytes"]]
            f.write(b"\0" * ((-f.tell()) % TRUNK_ALIGN))
            file_off, pos, ts = f.tell(), 0, {}
            for name, t in sorted(lay["tensors"].items(), key=lambda kv: kv[1]["off"]):
                b = run[t["off"]:t["off"] + t["nbytes"]]
                shape = t.get("shape", [])
                if t["dtype"] == "BF16" and len(shape) == 2:
                    u = np.frombuffer(b, np.uint16).reshape(shape)
                    enc = quant_rows_int8((u.astype(np.uint32) << 16).view(np.float32)).tobytes()
                    ts[name] = {"off": pos, "nbytes": len(enc), "dtype": "I8R", "shape": shape}
                    f.write(enc)
                    pos += len(enc)
                else:
                    ts[name] = {"off": pos, "nbytes": len(b), "dtype": t["dtype"], "shape": shape}
                    f.write(b)
                    pos += len(b)
            f.write(b"\0" * ((-f.tell()) % TRUNK_ALIGN))
            nl = {k: v for k, v in lay.items() if k not in ("file_off", "nbytes", "tensors")}
            nl.update({"file_off": file_off, "nbytes": (pos + TRUNK_ALIGN - 1) & ~(TRUNK_ALIGN - 1), "tensors": ts})
            new["layers"].append(nl)
    with open(os.path.join(out, "trunk.json"), "w") as f:
        json.dump(new, f)
    return new
