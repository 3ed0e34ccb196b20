"""Routed experts from safetensors shards into pool-format device runs (k3c_expert_upload):
byte-equal to packing the same expert from its arrays, for contiguous (O_DIRECT), reordered
and scattered runs, and usable by the tensor-core decode."""
import numpy as np
import pytest

from ckpt_util import build_checkpoint
from conftest import maxrel

pytestmark = pytest.mark.gpu


def test_upload_matches_pack(k3, tmp_path):
    import torch
    dev = torch.device("cuda:0")
    H, I = 256, 128
    want = build_checkpoint(str(tmp_path), k3.synth.rng(7), H, I)
    ck = k3.Checkpoint(str(tmp_path))
    rb = k3.pool_run_bytes(H, I)
    for (layer, expert), (_, e) in want.items():
        r = ck.expert_ref(layer, expert)
        payload = torch.from_numpy(ck.read_expert(r).copy()).pin_memory()
        staging = torch.empty(r.nbytes, dtype=torch.uint8, device=dev)
        got = torch.empty(rb, dtype=torch.uint8, device=dev)
        ck.upload(r, payload, got, staging)
        ref = torch.empty(rb, dtype=torch.uint8, device=dev)
        k3.pool_pack(ref, k3.DeviceExpert.from_host(e, dev).q(), H, I)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), (layer, expert)


def test_decode_from_checkpoint_runs(k3, ora, tmp_path):
    """A tensor-core decode layer whose arena is filled from the checkpoint files."""
    import torch
    dev = torch.device("cuda:0")
    H, I, K = 256, 128, 2
    want = build_checkpoint(str(tmp_path), k3.synth.rng(8), H, I)
    keys = [(1, 0), (1, 1), (1, 2), (2, 0)]
    ck = k3.Checkpoint(str(tmp_path))
    rb = k3.pool_run_bytes(H, I)
    arena = torch.empty(len(keys) * rb, dtype=torch.uint8, device=dev)
    for i, (layer, expert) in enumerate(keys):
        r = ck.expert_ref(layer, expert)
        payload = torch.from_numpy(ck.read_expert(r).copy())
        staging = torch.empty(r.nbytes, dtype=torch.uint8, device=dev)
        ck.upload(r, payload, arena[i * rb:(i + 1) * rb], staging)
        torch.cuda.synchronize()
    g = k3.synth.rng(9)
    wf, wb = k3.synth.router_weights(g, len(keys), H)
    wf = (wf * 20).astype(np.float32)
    wb = k3.synth.bf16_bits(wf)
    xf, xb = k3.synth.activations(g, 4, H)
    run_of = torch.arange(len(keys), dtype=torch.int32, device=dev)
    W = torch.from_numpy(wb.view(np.int16)).to(dev).view(torch.bfloat16)
    layer = k3.PoolMoeLayer(arena, len(keys), run_of, -1, W, None, H, I, K)
    out, idx, _ = layer.decode(torch.from_numpy(xb.view(np.int16)).to(dev))
    experts = [want[k][1] for k in keys]
    ref, ridx, _ = ora.moe_layer(xf, k3.synth.bf16_to_f32(wb), None, experts, None, H, I, K)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert maxrel(out.cpu().numpy(), ref) < 2e-2


def test_latent_layer_from_an_int8_draft_trunk(k3, ora, tmp_path):
    """The draft model's layer fed from a packed int8 trunk (the I8R tensors tools/int8_trunk.py
    writes, read by k3c_trunk_*): its down/up/shared matrices packed for the int8 tensor-core
    GEMV, the layer within 2e-2 of the oracle's k3_moe on the same int8 rows, routing exact."""
    import torch
    import ckpt_util as ck
    from conftest import maxrel
    g = k3.synth.rng(808)
    lay = k3.synth.latent_layer(g, 512, 256, 128, 16, 4, n_shared=1, wdt=1)
    names = {k: f"language_model.model.layers.0.block_sparse_moe.{k}.weight" for k in ("down", "up", "sh1", "sh3", "sh2")}
    ck.write_bf16_trunk(str(tmp_path / "bf16"), [[(names[k], lay[k]) for k in names]])
    ck.int8_trunk(str(tmp_path / "bf16"), str(tmp_path / "i8"))
    tr = k3.Trunk(str(tmp_path / "i8"))
    i8 = dict(lay, wdt=2)
    for k, n in names.items():
        t = tr.find(0, n)
        assert t.dtype == k3.DT_I8R
        i8[k] = tr.read(t).reshape(int(t.shape[0]), 4 + int(t.shape[1]))
    mat, keep = tr.q8_mat(0, names["down"], "cuda")
    wq, ws, ldw = k3.q8_pack(torch.from_numpy(i8["down"]).cuda(), 512, 256)
    assert torch.equal(keep[0], wq) and torch.equal(keep[1], ws) and mat.ldw == ldw
    x = g.standard_normal((5, 512), dtype=np.float32)
    want, widx, _ = ora.moe_latent(x, i8)
    out, idx, _ = k3.LatentMoeLayer.from_host(i8, "cuda").decode(torch.from_numpy(x).cuda())
    assert np.array_equal(idx.cpu().numpy(), widx)
    assert maxrel(out.cpu().numpy(), want) < 2e-2
    tr.close()
