"""Environments, rewards, schedules, image preprocessing, prompt builders and metric summaries (CPU).

Golden values are computed by hand from the formulas (haversine with R = 6371 km, exp(-d / tau) kernels,
the smart-resize rounding rules, the softmax cut-offs of top-k / top-p), not read back from the code.
"""

import math

import numpy as np
import pytest
import torch

from vlmrl.envs import base as envbase
from vlmrl.envs import geospot as G
from vlmrl.envs.nlvr2 import NLVR2Env, NLVR2Sample, parse_binary
from vlmrl.envs.schedule import DEFAULT_SCHEDULE, prepare_weight_schedule, weights_at
from vlmrl.envs.synthetic import SyntheticGeoEnv, SyntheticParityEnv, SyntheticTrueFalseEnv, sphere_point
from vlmrl.envs.vision_caption import VisionCaptionEnv
from vlmrl.utils import vlm
from vlmrl.utils.wandb import summarize_env_metrics


class CharTokenizer:
    """Token id = unicode code point; EOS = 0."""

    eos_token_id = 0

    def encode(self, text, add_special_tokens=False):
        return [ord(c) for c in text]

    def decode(self, ids, skip_special_tokens=True, clean_up_tokenization_spaces=False):
        return "".join(chr(i) for i in ids if i != 0)


# --------------------------------------------------------------------------- geospot parsing
def test_geospot_parse_key_value_lines():
    p = G.parse_response("City: Paris\nRegion: Ile-de-France\nCountry: France\nLatitude: 48.8566\nLongitude: 2.3522")
    assert (p.city, p.region, p.country) == ("Paris", "Ile-de-France", "France")
    assert p.coords == G.Coords(48.8566, 2.3522) and p.format_valid


def test_geospot_parse_markdown_aliases_first_wins_and_comma_decimal():
    p = G.parse_response("- City: **Lyon**\n* State: Auvergne\nCity: Other\n- Lat: 45,76\n- Lon: 4.83\nCountry: FR")
    assert p.city == "Lyon"              # emphasis stripped from the value; first occurrence wins
    assert p.region == "Auvergne"        # "state" is a region alias
    assert p.country == "FR"
    assert p.coords == G.Coords(45.76, 4.83)   # decimal comma accepted
    # as in the reference, a key must start with a letter: an emphasised key is not a key line
    assert G.parse_response("**City**: Lyon\nCountry: FR").city is None


def test_geospot_parse_delimited_fallback():
    p = G.parse_response("Paris, Ile-de-France, France, 48.85, 2.35")
    assert (p.city, p.region, p.country) == ("Paris", "Ile-de-France", "France")
    assert p.coords == G.Coords(48.85, 2.35)
    # a trailing pair outside [-90, 90] x [-180, 180] is not taken as coordinates
    q = G.parse_response("Paris, France, 123.0, 500.0")
    assert q.coords is None


def test_geospot_parse_empty_and_prose():
    assert not G.parse_response("").format_valid
    p = G.parse_response("I think this is somewhere in Europe")
    assert p.coords is None and not p.format_valid


# --------------------------------------------------------------------------- geospot reward
def test_haversine_golden_distances():
    # one degree of longitude on the equator = R * pi / 180
    assert G.haversine_km(G.Coords(0, 0), G.Coords(0, 1)) == pytest.approx(6371 * math.pi / 180, rel=1e-9)
    # antipodes = half the circumference
    assert G.haversine_km(G.Coords(0, 0), G.Coords(0, 180)) == pytest.approx(6371 * math.pi, rel=1e-9)
    # Paris -> London: closed-form great-circle distance with R = 6371 km
    p1, l1, p2, l2 = map(math.radians, (48.8566, 2.3522, 51.5074, -0.1278))
    a = math.sin((p2 - p1) / 2) ** 2 + math.cos(p1) * math.cos(p2) * math.sin((l2 - l1) / 2) ** 2
    want = 2 * 6371 * math.asin(math.sqrt(a))
    assert G.haversine_km(G.Coords(48.8566, 2.3522), G.Coords(51.5074, -0.1278)) == pytest.approx(want, rel=1e-9)
    assert 340 < want < 347


def _geocoder():
    return G.StaticGeocoder({
        "France": (46.6, 2.2), "Germany": (51.1, 10.4),
        "Ile-de-France, France": (48.7, 2.5), "Bavaria, Germany": (48.9, 11.4),
        "Paris, Ile-de-France, France": (48.8566, 2.3522), "Munich, Bavaria, Germany": (48.1351, 11.582),
    })


def test_geospot_reward_hierarchical_kernel():
    truth = G.Location("Paris", "Ile-de-France", "France", G.Coords(48.8566, 2.3522))
    cfg = G.RewardConfig()
    exact = G.parse_response("City: Paris\nRegion: Ile-de-France\nCountry: France\nLatitude: 48.8566\nLongitude: 2.3522")
    r = G.compute_reward(truth, exact, cfg, _geocoder())
    assert r.reward == pytest.approx(1.0) and r.within_tolerance and r.active_weight_sum == 4.0

    wrong = G.parse_response("City: Munich\nRegion: Bavaria\nCountry: Germany\nLatitude: 48.1351\nLongitude: 11.582")
    r = G.compute_reward(truth, wrong, cfg, _geocoder())
    d_c = G.haversine_km(G.Coords(46.6, 2.2), G.Coords(51.1, 10.4))
    d_r = G.haversine_km(G.Coords(48.7, 2.5), G.Coords(48.9, 11.4))
    d_t = G.haversine_km(G.Coords(48.8566, 2.3522), G.Coords(48.1351, 11.582))
    want = (math.exp(-d_c / 2000) + math.exp(-d_r / 500) + math.exp(-d_t / 100) + math.exp(-d_t / 25)) / 4
    assert r.reward == pytest.approx(want, rel=1e-9)
    assert not r.within_tolerance


def test_geospot_reward_drops_missing_fields_and_unparseable_scores_zero():
    truth = G.Location("Paris", "Ile-de-France", "France", G.Coords(48.8566, 2.3522))
    coords_only = G.parse_response("Latitude: 48.8566\nLongitude: 3.3522")
    r = G.compute_reward(truth, coords_only, G.RewardConfig(), _geocoder())
    d = G.haversine_km(truth.coords, G.Coords(48.8566, 3.3522))
    assert r.active_weight_sum == 1.0                       # only the coordinate field has a distance
    assert r.reward == pytest.approx(math.exp(-d / 25))
    junk = G.compute_reward(truth, G.parse_response("no idea"), G.RewardConfig(), _geocoder())
    assert junk.reward == 0.0 and junk.active_weight_sum == 0.0


def test_geospot_curriculum_stage_weights():
    stages = {s.name: s for s in G.DEFAULT_CURRICULUM}
    cfg = G.stage_reward_config(G.RewardConfig(), stages["region"])
    assert cfg.field_weights.coords == pytest.approx(max(0.0, 0.5 * 0.4))
    cfg = G.stage_reward_config(G.RewardConfig(), stages["full"])
    assert cfg.field_weights.coords == pytest.approx(0.4)
    env = G.GeospotEnv(CharTokenizer(), samples=[G.Sample(0, "missing.jpg", G.Location("", "", "", G.Coords(0, 0)))],
                       geocoder=G.StaticGeocoder())
    env._load_image = lambda sample: np.zeros((32, 32, 3), np.uint8)
    seen = []
    for _ in range(1001):
        st, _ = env.reset(0)
        seen.append(st.stage.name)
    assert seen[0] == "country_coarse" and seen[100] == "country" and seen[300] == "region"
    assert seen[600] == "city" and seen[1000] == "full"


def test_geospot_env_step_reward_and_info():
    truth = G.Location("Paris", "Ile-de-France", "France", G.Coords(48.8566, 2.3522))
    env = G.GeospotEnv(CharTokenizer(), samples=[G.Sample(0, "x.jpg", truth)], geocoder=_geocoder())
    env._load_image = lambda sample: np.zeros((32, 32, 3), np.uint8)
    st, prompt = env.reset(0)
    assert "Latitude" in prompt.question
    text = "City: Paris\nRegion: Ile-de-France\nCountry: France\nLatitude: 48.8566\nLongitude: 2.3522"
    _, out, reward, done, info = env.step(st, CharTokenizer().encode(text) + [0, 65, 66])  # tokens after EOS dropped
    assert done and out == [] and reward == pytest.approx(1.0)
    assert info["parsed"]["city"] == "Paris" and info["stage"] == "country_coarse"


# --------------------------------------------------------------------------- other environments
def test_nlvr2_parse_and_reward():
    assert parse_binary("True") and parse_binary("yes, it is") and not parse_binary("False.")
    assert not parse_binary("no")
    assert not parse_binary("true or false")          # both words: undecided -> False
    samples = [NLVR2Sample("There are two dogs.", None, None, True), NLVR2Sample("One cat.", None, None, False)]
    env = NLVR2Env(CharTokenizer(), samples=samples)
    st, prompt = env.reset(0)
    assert prompt.statement == "There are two dogs."
    assert env.step(st, CharTokenizer().encode("True"))[2] == 1.0
    st, _ = env.reset(1)
    assert env.step(st, CharTokenizer().encode("True"))[2] == 0.0
    assert env.num_tasks == 2


def test_vision_caption_keyword_fraction():
    env = VisionCaptionEnv(CharTokenizer())
    st, prompt = env.reset(0)
    kws = list(st.sample.keywords)
    assert kws and prompt.keywords == st.sample.keywords
    half = " ".join(kws[: max(1, len(kws) // 2)])
    _, _, r, _, info = env.step(st, CharTokenizer().encode(half))
    assert r == pytest.approx(info["hits"] / len(kws)) and info["hits"] >= max(1, len(kws) // 2)
    assert env.step(st, CharTokenizer().encode("zzzz"))[2] == 0.0


def test_vision_caption_ships_its_demo_images():
    """Every caption task's image exists in the package (no random placeholder) and preprocesses."""
    from vlmrl.models.qwen3vl.config import get_preset
    from vlmrl.utils.vlm import preprocess_image

    env = VisionCaptionEnv(CharTokenizer())
    spec = get_preset("tiny")
    seen = set()
    for i in range(env.num_tasks):
        st, prompt = env.reset(i)
        assert prompt.image is None, st.sample.image_path   # the file is there
        if st.sample.image_path in seen:
            continue
        seen.add(st.sample.image_path)
        v = spec.vision
        rows, grid = preprocess_image(st.sample.image_path, patch_size=v.patch_size,
                                      spatial_merge_size=v.spatial_merge_size,
                                      temporal_patch_size=v.temporal_patch_size, max_pixels=64 * 64 * 4)
        assert rows.shape[0] == int(grid.prod()) and torch.isfinite(rows).all()
    assert len(seen) == 7


def test_synthetic_envs_rewards():
    tok = CharTokenizer()
    par = SyntheticParityEnv(tok, num_tasks=4)
    st, _ = par.reset(0)
    assert par.step(st, [4, 7])[2] == 1.0 and par.step(st, [7, 4])[2] == 0.0
    tf = SyntheticTrueFalseEnv(tok, true_id=11, false_id=12, num_tasks=8)
    labels = []
    for i in range(8):
        st, _ = tf.reset(i)
        labels.append(st.target)
        want = 11 if st.target else 12
        assert tf.step(st, [want])[2] == 1.0 and tf.step(st, [23 - want])[2] == 0.0
    st2, _ = tf.reset(3)
    assert st2.target == labels[3]                      # labels are a function of (seed, index)
    geo = SyntheticGeoEnv(tok, num_tasks=4)
    st, _ = geo.reset(1)
    c = st.target
    _, _, r, _, info = geo.step(st, tok.encode(f"Latitude: {c.lat}\nLongitude: {c.lon}"))
    assert r == pytest.approx(1.0, abs=1e-6) and info["coords_within_tolerance"] == 1.0
    _, _, r0, _, _ = geo.step(st, tok.encode("no coordinates"))
    assert r0 == 0.0


def test_sphere_point_is_uniform_on_the_sphere():
    rng = np.random.default_rng(0)
    pts = [sphere_point(rng) for _ in range(20000)]
    z = np.array([math.sin(math.radians(p.lat)) for p in pts])
    # uniform on the sphere <=> sin(latitude) uniform on [-1, 1]: mean 0, variance 1/3
    assert abs(z.mean()) < 0.02 and abs(z.var() - 1 / 3) < 0.02


# --------------------------------------------------------------------------- schedule, registry
def test_weight_schedule_defaults_and_custom_entries():
    target = {"country": 0.2, "region": 0.3, "city": 0.5}
    s = prepare_weight_schedule(None, target)
    assert list(s) == sorted(DEFAULT_SCHEDULE)
    assert weights_at(s, 0)["weights"] == {"country": 0.2, "region": 0.0, "city": 0.0}
    assert weights_at(s, 2000)["weights"] == {"country": 0.2, "region": 0.3, "city": 0.0}
    assert weights_at(s, 10 ** 6)["weights"] == target
    c = prepare_weight_schedule({"5": {"label": "Warm", "weights": {"region": 1.0}}, "bad": "x"}, target)
    assert list(c) == [5] and c[5]["label"] == "warm"
    assert c[5]["weights"] == {"country": 0.2, "region": 1.0, "city": 0.0}
    assert prepare_weight_schedule({"bad": 3}, target) == {0: {"label": "full", "weights": target}}


def test_registry_aliases_clean_action_and_step_list():
    assert envbase._ENV_REGISTRY["truefalse"] == envbase._ENV_REGISTRY["nlvr2"]
    assert envbase._ENV_REGISTRY["caption"] == envbase._ENV_REGISTRY["vision_caption"] == envbase._ENV_REGISTRY["vision"]
    with pytest.raises(ValueError):
        envbase.create_env("no_such_env", CharTokenizer())
    env = envbase.create_env("Synthetic_Parity", CharTokenizer(), num_tasks=2)
    assert isinstance(env, SyntheticParityEnv)
    assert envbase.BaseEnv.clean_action([5, 7, 0, 9], 0) == [5, 7, 0]
    states = [env.reset(i)[0] for i in range(2)]
    _, outs, rewards, dones, info = env.step_list(states, [[2], [3]])
    assert rewards == [1.0, 0.0] and dones == [True, True] and info["first_token"] == [2, 3]
    with pytest.raises(ValueError):
        env.step_list(states, [[2]])


# --------------------------------------------------------------------------- image + prompt utilities
def test_smart_resize_rounding_rules():
    big = 10 ** 9
    assert vlm.smart_resize(448, 448, factor=32, min_pixels=3136, max_pixels=big) == (448, 448)
    assert vlm.smart_resize(100, 1000, factor=32, min_pixels=1, max_pixels=big) == (96, 992)
    # over the pixel budget: scale by sqrt(h*w / max), floor to the factor
    assert vlm.smart_resize(2000, 2000, factor=32, min_pixels=1, max_pixels=1003520) == (992, 992)
    # under it: scale up, ceil to the factor
    assert vlm.smart_resize(10, 10, factor=32, min_pixels=3136, max_pixels=big) == (64, 64)
    with pytest.raises(ValueError):
        vlm.smart_resize(1, 300, factor=32, min_pixels=1, max_pixels=big)


def test_preprocess_image_normalisation_and_merge_order():
    # patch (ph, pw) of a 64x64 image is filled with the value 10*pw + ph (red channel)
    img = np.zeros((64, 64, 3), np.uint8)
    for ph in range(4):
        for pw in range(4):
            img[16 * ph:16 * ph + 16, 16 * pw:16 * pw + 16, 0] = 10 * pw + ph
    rows, grid = vlm.preprocess_image(img, patch_size=16, spatial_merge_size=2, temporal_patch_size=2,
                                      min_pixels=1, max_pixels=10 ** 9)
    assert grid.tolist() == [[1, 4, 4]] and tuple(rows.shape) == (16, 3 * 2 * 16 * 16)
    red = rows[:, 0].numpy() * vlm.CLIP_STD[0] + vlm.CLIP_MEAN[0]
    got = np.rint(red * 255).astype(int)
    # rows walk 2x2 merge windows in raster order, and the 4 patches of a window in raster order
    want = [10 * pw + ph for hb in range(2) for wb in range(2) for hm in range(2) for wm in range(2)
            for ph, pw in [(2 * hb + hm, 2 * wb + wm)]]
    assert got.tolist() == want
    # both temporal copies of a frame are identical; the green channel starts at 2 * 16 * 16
    assert torch.equal(rows[:, :256], rows[:, 256:512])
    assert rows[0, 512].item() == pytest.approx((0 - vlm.CLIP_MEAN[1]) / vlm.CLIP_STD[1], rel=1e-5)


def test_prompt_builders_and_extract_assistant():
    p = vlm.chat_prompt_with_image(3, "Where?")
    assert p == ("<|im_start|>user\n<|vision_start|><|image_pad|><|image_pad|><|image_pad|><|vision_end|>"
                 "Where?<|im_end|>\n<|im_start|>assistant\n")
    two = vlm.chat_prompt_with_images([1, 2], "Q")
    assert two.count("<|vision_start|>") == 2 and two.count("<|image_pad|>") == 3
    assert vlm.extract_assistant(p + "Paris<|im_end|>") == "Paris"
    assert vlm.extract_assistant(p + "unterminated") == "unterminated"
    assert vlm.extract_assistant("no assistant turn") is None


def test_top_k_top_p_mask_golden():
    logits = torch.tensor([[0.0, 1.0, 2.0, 3.0, 4.0]])
    m = vlm.mask_logits_topk_topp(logits, top_k=3, top_p=None)
    assert (m[0, 2:] == logits[0, 2:]).all() and (m[0, :2] == vlm.MASK_VALUE).all()
    # softmax over the top 3 (4, 3, 2) = (0.665, 0.245, 0.090): p = 0.95 keeps two, p = 0.5 keeps the first only
    m = vlm.mask_logits_topk_topp(logits, top_k=3, top_p=0.95)
    assert (m[0, 3:] == logits[0, 3:]).all() and (m[0, :3] == vlm.MASK_VALUE).all()
    m = vlm.mask_logits_topk_topp(logits, top_k=3, top_p=0.5)
    assert m[0, 4] == 4.0 and (m[0, :4] == vlm.MASK_VALUE).all()
    # top-p only (full-vocabulary nucleus)
    m = vlm.mask_logits_topk_topp(logits, top_k=None, top_p=0.95)
    assert (m[0, 3:] == logits[0, 3:]).all() and (m[0, :3] == vlm.MASK_VALUE).all()


def test_env_metric_summary():
    out = summarize_env_metrics({"distance_km": [10.0, 30.0, 200.0, 1000.0], "format_ok": [1, 0, 1, 1],
                                 "has_coords": [1, 1, 1, 0], "coords_within_tolerance": [1, 0, 0, 0],
                                 "stage_idx": [0, 2], "response": ["ignored"] * 4})
    assert out["env/within_25km"] == 0.25 and out["env/within_100km"] == 0.5 and out["env/within_500km"] == 0.75
    assert out["env/distance_p50"] == pytest.approx(115.0) and out["env/format_ok"] == 0.75
    assert out["env/stage_idx"] == 2.0 and "env/response" not in out
    # weights 1, 2 for (has_coords, coords_within_tolerance) in that order
    assert out["env/coord_quality_score"] == pytest.approx((0.75 * 1 + 0.25 * 2) / 3)
