"""The reference's own Qwen3-VL vision tower (``vision_arch="reference"``) against an independent oracle.

The oracle below restates the reference tower's computation (reference ``models/qwen3vl/vision.py``:
patch Dense without bias :33-41, rotary table :21-30 and its use :69-77/:280-284, padded window index
:233-272, per-window attention :79-106, RMSNorm + biased SwiGLU blocks :120-144, mergers with tanh-GELU
:147-175, window unshuffle :324-327) in plain fp32 PyTorch, reading its weights by the reference's Flax
names from ``units_to_flax`` — so the test checks the parameter naming and the math together.
"""

from dataclasses import replace

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from vlmrl.models.qwen3vl.api import Qwen3VLModel
from vlmrl.models.qwen3vl.config import get_preset, spec_from_config, spec_to_config
from vlmrl.models.qwen3vl.params import flax_to_units, init_params, units_to_flax
from vlmrl.models.qwen3vl.weights import hf_state_dict_to_units, units_to_hf_state_dict


def _spec(window_size: int):
    spec = get_preset("tiny", vision_arch="reference")
    return replace(spec, vision=replace(spec.vision, window_size=window_size, num_position_embeddings=None))


def _rms(x, w, eps=1e-6):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _dense(tree, x):
    return x @ torch.as_tensor(tree["kernel"]) + (torch.as_tensor(tree["bias"]) if "bias" in tree else 0.0)


def _window_index(grids, merge, window, patch):
    """The reference's padded window index (sentinel -100, then filtered)."""
    vw = window // merge // patch
    idx_all, cu, base = [], [0], 0
    for t, h, w in grids:
        gh, gw = h // merge, w // merge
        index = np.arange(t * gh * gw).reshape(t, gh, gw)
        ph, pw = (vw - gh % vw) % vw, (vw - gw % vw) % vw
        nh, nw = (gh + ph) // vw, (gw + pw) // vw
        pad = np.pad(index, ((0, 0), (0, ph), (0, pw)), constant_values=-100)
        pad = pad.reshape(t, nh, vw, nw, vw).transpose(0, 1, 3, 2, 4).reshape(t, nh * nw, vw, vw)
        seqlens = (pad != -100).sum(axis=(2, 3)).reshape(-1)
        flat = pad.reshape(-1)
        idx_all.append(flat[flat != -100] + base)
        cu.extend(list(np.cumsum(seqlens) * merge * merge + cu[-1]))
        base += t * gh * gw
    cu = np.asarray(cu)
    keep = np.concatenate([[True], cu[1:] != cu[:-1]])
    return np.concatenate(idx_all), cu[keep]


def _oracle(spec, tree, pixels, grids):
    v = spec.vision
    Hv, nh, m = v.hidden_size, v.num_heads, v.spatial_merge_size
    D = Hv // nh
    unit = m * m
    vis = tree["visual"]
    x = pixels.float() @ torch.as_tensor(vis["patch_embed"]["proj"]["kernel"])
    # rotary: (row, col) in merge-window order, D/2 frequencies, angles [row*f | col*f]
    pos = []
    for t, h, w in grids:
        hp = np.arange(h)[:, None].repeat(w, 1).reshape(h // m, m, w // m, m).transpose(0, 2, 1, 3).reshape(-1)
        wp = np.arange(w)[None, :].repeat(h, 0).reshape(h // m, m, w // m, m).transpose(0, 2, 1, 3).reshape(-1)
        pos.append(np.tile(np.stack([hp, wp], -1), (t, 1)))
    pos = torch.as_tensor(np.concatenate(pos))
    rdim = D // 2
    inv = 1.0 / (10000.0 ** (torch.arange(rdim, dtype=torch.float32) / rdim))
    rot = (pos.float()[..., None] * inv).reshape(pos.shape[0], -1)  # [N, D]
    widx, cu_w = _window_index(grids, m, v.window_size, v.patch_size)
    N = x.shape[0]
    x = x.reshape(N // unit, unit, -1)[widx].reshape(N, -1)
    rot = rot.reshape(N // unit, unit, -1)[widx].reshape(N, -1)
    cos, sin = torch.cos(rot)[:, None], torch.sin(rot)[:, None]

    def rope(t):
        t1, t2 = t[..., :rdim], t[..., rdim:]
        return t * cos + torch.cat([-t2, t1], -1) * sin

    cu_full = np.concatenate([[0], np.cumsum([t * h * w for t, h, w in grids])])
    deep_idx = list(v.deepstack_visual_indexes)
    deep = []
    for j in range(v.depth):
        blk = vis[f"blocks_{j}"]
        cu = cu_full if j in set(v.fullatt_block_indexes) else cu_w
        hn = _rms(x, torch.as_tensor(blk["norm1"]["weight"]))
        q, k, vv = _dense(blk["attn"]["qkv"], hn).reshape(N, 3, nh, D).unbind(1)
        q, k = rope(q), rope(k)
        o = torch.empty_like(q)
        for s, e in zip(cu[:-1], cu[1:]):
            sc = torch.einsum("qhd,khd->hqk", q[s:e], k[s:e]) * D ** -0.5
            o[s:e] = torch.einsum("hqk,khd->qhd", sc.softmax(-1), vv[s:e])
        x = x + _dense(blk["attn"]["proj"], o.reshape(N, Hv))
        hn = _rms(x, torch.as_tensor(blk["norm2"]["weight"]))
        mlp = blk["mlp"]
        x = x + _dense(mlp["down_proj"], F.silu(_dense(mlp["gate_proj"], hn)) * _dense(mlp["up_proj"], hn))
        if j in deep_idx:
            mg = vis[f"deepstack_mergers_{deep_idx.index(j)}"]
            h2 = _rms(x.reshape(-1, unit * Hv), torch.as_tensor(mg["norm"]["weight"]))
            deep.append(_dense(mg["linear2"], F.gelu(_dense(mg["linear1"], h2), approximate="tanh")))
    mg = vis["merger"]
    h2 = _rms(x, torch.as_tensor(mg["norm"]["weight"])).reshape(-1, unit * Hv)
    merged = _dense(mg["linear2"], F.gelu(_dense(mg["linear1"], h2), approximate="tanh"))
    rev = torch.as_tensor(np.argsort(widx))
    return merged[rev], [d[rev] for d in deep]


@pytest.mark.parametrize("window_size,grids", [(32, [(1, 8, 12)]), (64, [(1, 6, 10)]), (64, [(2, 4, 8)])])
def test_reference_tower_matches_oracle(window_size, grids):
    spec = _spec(window_size)
    units = init_params(spec, seed=5)
    v = spec.vision
    # larger draws than the init's so that every block changes the activations visibly
    lay_units = {k: t.clone() for k, t in units.items()}
    g = torch.Generator().manual_seed(3)
    lay_units["visual"] += 0.05 * torch.randn(lay_units["visual"].shape, generator=g)
    model = Qwen3VLModel(spec, units=lay_units, dtype=torch.float32)
    n = sum(t * h * w for t, h, w in grids)
    pix = torch.randn(n, v.patch_volume, generator=g)
    emb = model.encode_vision(pix, grids)
    tree = units_to_flax(spec, lay_units)
    want, want_deep = _oracle(spec, tree, pix, grids)
    assert emb.tokens.shape == want.shape
    torch.testing.assert_close(emb.tokens, want, rtol=2e-4, atol=2e-4)
    assert len(emb.deepstack) == len(v.deepstack_visual_indexes) == len(want_deep)
    for a, b in zip(emb.deepstack, want_deep):
        torch.testing.assert_close(a, b, rtol=2e-4, atol=2e-4)


def test_reference_tower_tree_names_and_round_trips():
    spec = _spec(32)
    units = init_params(spec, seed=9)
    tree = units_to_flax(spec, units)
    vis = tree["visual"]
    assert set(vis["blocks_0"]["mlp"]) == {"gate_proj", "up_proj", "down_proj"}
    assert set(vis["blocks_0"]["norm1"]) == {"weight"}
    assert set(vis["merger"]) == {"norm", "linear1", "linear2"}
    assert set(vis["deepstack_mergers_0"]["norm"]) == {"weight"}
    assert vis["deepstack_mergers_0"]["norm"]["weight"].shape == (4 * spec.vision.hidden_size,)
    assert set(vis["patch_embed"]["proj"]) == {"kernel"} and "pos_embed" not in vis
    back = flax_to_units(spec, tree, strict=True)
    for k in units:
        assert torch.equal(back[k], units[k]), k
    sd = units_to_hf_state_dict(spec, units)
    assert "model.visual.deepstack_merger_list.0.norm.weight" in sd
    back = hf_state_dict_to_units(spec, sd)
    torch.testing.assert_close(back["visual"], units["visual"], rtol=0, atol=0)
    spec2 = spec_from_config(spec_to_config(spec))
    assert spec2.vision_arch == "reference"
    assert spec2.vision.window_size == 32 and tuple(spec2.vision.fullatt_block_indexes) == (1,)
