"""Environment <-> model glue: prompt preparation, batched episode collection, training batches.

Counterpart of reference ``core/rollout.py:46-426``, batched instead of serial:

* ``prepare_prompts`` turns observations into token ids + one vision encode for
  every image of the batch.  Same-size uint8 images (the synthetic envs) are
  copied to the GPU through one pinned buffer and patchified there; other
  images go through ``preprocess_image`` (PIL bicubic, CPU).  Single-image
  observations (``image``/``image_path`` + ``question``) use the chat template
  of ``chat_prompt_with_image``; two-image observations (``image_left``,
  ``image_right``, ``statement``) use ``chat_prompt_with_images`` with the
  question ``"Look at the two images. {statement}"``; synthetic observations
  carry token ids directly (vision block per image + prompt ids).
* ``collect_episodes`` resets ``groups_per_batch`` tasks, samples
  ``group_size`` responses per task in ONE batched generate call (the prompt is
  prefilled once per group and its KV cache replicated), scores them with
  ``env.step_list`` and returns an ``EpisodeBatch``.
* ``episodes_to_training_batch`` builds the packed training batch (inputs
  ``s[:-1]``, targets ``s[1:]``, loss rows on the action tokens) and the
  ``Rollout`` record.  Actions are cut after the first EOS (inclusive), so
  EOS padding is not trained on.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from vlmrl.core.batching import pack_sequences
from vlmrl.core.sampling import Generator
from vlmrl.core.types import Rollout, SamplingConfig
from vlmrl.envs.base import BaseEnv, BaseState
from vlmrl.models.qwen3vl.model import VisionEmbeddings
from vlmrl.utils.vlm import (DEFAULT_MAX_PIXELS, DEFAULT_MIN_PIXELS, chat_prompt_with_image, chat_prompt_with_images,
                             preprocess_image, smart_resize)


@dataclass
class PreparedPrompt:
    prompt_tokens: np.ndarray
    prompt_length: int
    grids: List[Tuple[int, int, int]]
    prompt_text: str = ""


@dataclass
class Episode:
    state: BaseState
    observation: Any
    prompt_text: str
    prompt_tokens: np.ndarray
    prompt_length: int
    full_tokens: np.ndarray
    full_logprobs: np.ndarray
    action_tokens: List[int]
    action_logprobs: np.ndarray
    action_length: int
    generated_text: str
    grids: List[Tuple[int, int, int]]
    reward: float
    done: bool
    info: Dict[str, Any] = field(default_factory=dict)
    group_id: int = 0


@dataclass
class EpisodeBatch:
    episodes: List[Episode]
    raw_info: Dict[str, List[Any]]
    vision: Optional[VisionEmbeddings] = None       # per episode, in episode order
    group_size: int = 1

    def subset(self, g0: int, g1: int, merge: int) -> "EpisodeBatch":
        """Groups [g0, g1) (episodes in (group, member) order) with their vision rows."""
        gs = max(1, self.group_size)
        eps = self.episodes[g0 * gs:g1 * gs]
        vis = self.vision
        if vis is not None:
            counts = [sum(_merged_count(g, merge) for g in ep.grids) for ep in self.episodes]
            start = int(sum(counts[:g0 * gs]))
            n = int(sum(counts[g0 * gs:g1 * gs]))
            vis = vis.select(torch.arange(start, start + n, device=vis.tokens.device))
        info = {k: v[g0 * gs:g1 * gs] for k, v in self.raw_info.items()} if self.raw_info else {}
        return EpisodeBatch(episodes=eps, raw_info=info, vision=vis, group_size=self.group_size)


def _images_of(obs) -> List[Any]:
    if hasattr(obs, "images"):
        return list(obs.images)
    if hasattr(obs, "image_left") and hasattr(obs, "image_right"):
        return [obs.image_left, obs.image_right]
    img = getattr(obs, "image", None)
    if img is None:
        img = getattr(obs, "image_path", None)
    if img is None:
        raise ValueError("Observation must expose `image` or `image_path` for vision sampling.")
    return [img]


def _gpu_ready(images: Sequence[Any], factor: int, min_px: int, max_px: int) -> bool:
    """All images are same-size uint8 HWC arrays that need no resize."""
    if not images or not all(isinstance(im, np.ndarray) and im.dtype == np.uint8 and im.ndim == 3 for im in images):
        return False
    h, w = images[0].shape[:2]
    if any(im.shape != images[0].shape for im in images):
        return False
    return smart_resize(h, w, factor=factor, min_pixels=min_px, max_pixels=max_px) == (h, w)


def encode_images(model, images: Sequence[Any], *, min_pixels: int = DEFAULT_MIN_PIXELS,
                  max_pixels: int = DEFAULT_MAX_PIXELS) -> Tuple[VisionEmbeddings, List[Tuple[int, int, int]]]:
    v = model.spec.vision
    factor = v.patch_size * v.spatial_merge_size
    if model.device.type == "cuda" and _gpu_ready(images, factor, min_pixels, max_pixels):
        host = torch.from_numpy(np.stack(images)).pin_memory()
        dev = host.to(model.device, non_blocking=True)
        emb = model.encode_images_uint8(dev)
        h, w = images[0].shape[:2]
        return emb, [(1, h // v.patch_size, w // v.patch_size)] * len(images)
    rows, grids = [], []
    for im in images:
        px, g = preprocess_image(im, patch_size=v.patch_size, spatial_merge_size=v.spatial_merge_size,
                                 temporal_patch_size=v.temporal_patch_size, min_pixels=min_pixels, max_pixels=max_pixels)
        rows.append(px)
        grids.append(tuple(int(x) for x in g[0].tolist()))
    emb = model.encode_vision(torch.cat(rows).to(model.device, model.dtype), grids)
    return emb, grids


def _merged_count(grid, merge: int) -> int:
    t, h, w = grid
    return int(t) * (int(h) // merge) * (int(w) // merge)


def prepare_prompts(model, tokenizer, observations: Sequence[Any], *, min_pixels: Optional[int] = None,
                    max_pixels: Optional[int] = None) -> Tuple[List[PreparedPrompt], VisionEmbeddings]:
    spec = model.spec
    merge = spec.vision.spatial_merge_size
    min_px = int(min_pixels) if min_pixels and min_pixels > 0 else DEFAULT_MIN_PIXELS
    max_px = int(max_pixels) if max_pixels and max_pixels > 0 else DEFAULT_MAX_PIXELS
    per_obs = [_images_of(o) for o in observations]
    flat = [im for ims in per_obs for im in ims]
    vision, grids = encode_images(model, flat, min_pixels=min_px, max_pixels=max_px)
    out: List[PreparedPrompt] = []
    gi = 0
    for obs, ims in zip(observations, per_obs):
        g = grids[gi:gi + len(ims)]
        gi += len(ims)
        counts = [_merged_count(x, merge) for x in g]
        if hasattr(obs, "prompt_ids") and getattr(obs, "question", None) is None:
            ids: List[int] = []
            for c in counts:
                ids += [spec.vision_start_token_id] + [spec.image_token_id] * c + [spec.vision_end_token_id]
            ids += [int(t) for t in np.asarray(obs.prompt_ids).reshape(-1)]
            text = ""
        else:
            if hasattr(obs, "statement") and len(ims) == 2:
                question = f"Look at the two images. {getattr(obs, 'statement', '')}"
            else:
                question = getattr(obs, "question", "") or ""
            text = chat_prompt_with_image(counts[0], question) if len(counts) == 1 else chat_prompt_with_images(counts, question)
            ids = list(tokenizer.encode(text, add_special_tokens=False))
        arr = np.asarray(ids, dtype=np.int64)
        out.append(PreparedPrompt(prompt_tokens=arr, prompt_length=len(arr), grids=list(g), prompt_text=text))
    return out, vision


def _vision_rows_per_prompt(prompts: Sequence[PreparedPrompt], merge: int) -> List[np.ndarray]:
    rows, off = [], 0
    for p in prompts:
        n = sum(_merged_count(g, merge) for g in p.grids)
        rows.append(np.arange(off, off + n))
        off += n
    return rows


def collect_episodes(env: BaseEnv, tokenizer, model, sampling_cfg: SamplingConfig, *, batch_size: int = 0,
                     groups_per_batch: int = 0, group_size: int = 1, seed: int = 0, task_offset: int = 0,
                     min_pixels: Optional[int] = None, max_pixels: Optional[int] = None,
                     max_sequence_length: Optional[int] = None, generator: Optional[Generator] = None,
                     row_offset: int = 0, **_: Any) -> EpisodeBatch:
    """Reset ``groups_per_batch`` tasks (or ``batch_size`` tasks with group_size 1) and sample ``group_size`` each."""
    G = int(groups_per_batch) if groups_per_batch else int(batch_size)
    gs = max(1, int(group_size))
    states, observations = [], []
    for g in range(G):
        s, o = env.reset(task_offset + g)
        states.append(s)
        observations.append(o)
    prompts, vision = prepare_prompts(model, tokenizer, observations, min_pixels=min_pixels, max_pixels=max_pixels)
    merge = model.spec.vision.spatial_merge_size
    gen = generator if generator is not None else Generator(model)
    res = gen.generate([p.prompt_tokens for p in prompts], [p.grids for p in prompts], vision, sampling_cfg,
                       seed=seed, row_offset=row_offset, group_size=gs)
    toks = res.tokens.cpu().numpy()
    lps = res.logprobs.cpu().numpy()
    lens = res.lengths.cpu().numpy()
    # episodes in (group, member) order
    ep_states, actions, meta = [], [], []
    for g in range(G):
        for j in range(gs):
            b = g * gs + j
            p = prompts[g]
            n = int(lens[b])
            if max_sequence_length is not None:
                n = max(0, min(n, int(max_sequence_length) - p.prompt_length))
            ep_states.append(states[g])
            actions.append(toks[b, :n].tolist())
            meta.append((g, b, n))
    _, _, rewards, dones, info = env.step_list(ep_states, actions)
    texts = [tokenizer.decode(a, skip_special_tokens=True) if tokenizer is not None else "" for a in actions]
    episodes: List[Episode] = []
    for i, (g, b, n) in enumerate(meta):
        p = prompts[g]
        act = np.asarray(actions[i], dtype=np.int64)
        alp = lps[b, :n].astype(np.float32)
        episodes.append(Episode(
            state=ep_states[i], observation=observations[g], prompt_text=p.prompt_text, prompt_tokens=p.prompt_tokens,
            prompt_length=p.prompt_length, full_tokens=np.concatenate([p.prompt_tokens, act]),
            full_logprobs=np.concatenate([np.zeros(p.prompt_length, np.float32), alp]), action_tokens=actions[i],
            action_logprobs=alp, action_length=n, generated_text=texts[i], grids=p.grids, reward=float(rewards[i]),
            done=bool(dones[i]), info={k: v[i] for k, v in info.items() if i < len(v)}, group_id=g))
    # vision rows of every episode (group members share their prompt's rows)
    rows = _vision_rows_per_prompt(prompts, merge)
    ep_rows = np.concatenate([rows[g] for g in range(G) for _ in range(gs)]) if G else np.zeros(0, np.int64)
    idx = torch.from_numpy(ep_rows).to(vision.tokens.device)
    return EpisodeBatch(episodes=episodes, raw_info=info, vision=vision.select(idx), group_size=gs)


def episodes_to_training_batch(model, episodes: Sequence[Episode], *, vision: Optional[VisionEmbeddings] = None,
                               pad_id: int = 0, max_sequence_length: Optional[int] = None, device=None):
    """-> (Rollout, PackedBatch).  ``vision`` must hold every episode's image rows in episode order."""
    if not episodes:
        raise ValueError("episodes_to_training_batch requires at least one episode.")
    spec = model.spec
    device = device or model.device
    seqs = [np.asarray(ep.full_tokens, dtype=np.int64) for ep in episodes]
    plens = np.asarray([ep.prompt_length for ep in episodes], dtype=np.int64)
    alens = np.asarray([ep.action_length for ep in episodes], dtype=np.int64)
    if max_sequence_length is not None:
        seqs = [s[:int(max_sequence_length)] for s in seqs]
    batch, counts = pack_sequences(spec, seqs, plens, [ep.grids for ep in episodes], vision, device=device)
    # sampler log-probs of exactly the scored rows (action tokens)
    samp = np.concatenate([np.asarray(ep.action_logprobs[:c], np.float32) for ep, c in zip(episodes, counts)])
    samp_t = torch.from_numpy(samp).to(device)
    rollout = Rollout(
        tokens=seqs, old_logprobs=samp_t.clone(), returns=torch.tensor([ep.reward for ep in episodes], dtype=torch.float32),
        mask_targets=torch.ones(len(samp), dtype=torch.float32, device=device), prompt_lens=plens, action_lens=alens,
        texts=[ep.generated_text for ep in episodes], group_ids=np.asarray([ep.group_id for ep in episodes]),
        sampler_logprobs=samp_t, token_counts=counts)
    return rollout, batch


def main(argv=None) -> List[float]:
    """Sample environment episodes without training (reference CLI, ``core/rollout.py:451-521``)."""
    import argparse

    from vlmrl.core.train import load_policy, resolve_pad_and_eos
    from vlmrl.envs.base import create_env
    from vlmrl.utils.rng import RngSeq
    from vlmrl.utils.tokenizer import load_tokenizer

    ap = argparse.ArgumentParser(description="Collect RL episodes using the unified sampler.")
    ap.add_argument("--model_dir", default="", type=str)
    ap.add_argument("--preset", default="", type=str, help="random-init architecture when model_dir has no weights")
    ap.add_argument("--env_name", required=True, type=str)
    ap.add_argument("--episodes", type=int, default=4)
    ap.add_argument("--batch_size", type=int, default=1)
    ap.add_argument("--group_size", type=int, default=1)
    ap.add_argument("--temperature", type=float, default=0.7)
    ap.add_argument("--top_p", type=float, default=0.9)
    ap.add_argument("--top_k", type=int, default=None)
    ap.add_argument("--max_new_tokens", type=int, default=64)
    ap.add_argument("--compat_refeed_last_token", action="store_true",
                    help="start decoding like the reference sampler (last prompt token decoded twice)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--min_pixels", type=int, default=-1)
    ap.add_argument("--max_pixels", type=int, default=-1)
    args = ap.parse_args(argv)
    dev = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    model, _ = load_policy(args.model_dir, args.preset, dev, torch.bfloat16 if dev.type == "cuda" else torch.float32,
                           seed=args.seed)
    tokenizer = load_tokenizer(args.model_dir or None, vocab_size=model.spec.text.vocab_size)
    env = create_env(args.env_name, tokenizer)
    pad_id, eos_id = resolve_pad_and_eos(tokenizer, model.spec)
    cfg = SamplingConfig(temperature=float(args.temperature),
                         top_p=float(args.top_p) if 0.0 < float(args.top_p) < 1.0 else None,
                         top_k=int(args.top_k) if args.top_k is not None and int(args.top_k) > 0 else None,
                         eos_id=eos_id, pad_id=pad_id, max_new_tokens=int(args.max_new_tokens),
                         compat_refeed_last_token=bool(args.compat_refeed_last_token))
    rng = RngSeq(int(args.seed))
    gen = Generator(model)
    remaining, taken, cursor = max(0, int(args.episodes)), 0, 0
    rewards: List[float] = []
    gs = max(1, int(args.group_size))
    while remaining > 0:
        take = max(1, min(int(args.batch_size), -(-remaining // gs)))
        eb = collect_episodes(env, tokenizer, model, cfg, groups_per_batch=take, group_size=gs, seed=rng.next(),
                              task_offset=cursor, generator=gen,
                              min_pixels=args.min_pixels if args.min_pixels > 0 else None,
                              max_pixels=args.max_pixels if args.max_pixels > 0 else None)
        cursor += take
        for ep in eb.episodes[:remaining]:
            rewards.append(float(ep.reward))
            resp = ep.generated_text.replace("\n", " ").strip()
            prompt = ep.prompt_text.strip().splitlines()[-1] if ep.prompt_text.strip() else ""
            keys = ", ".join(sorted(ep.info.keys())) if ep.info else "none"
            print(f"[episode {taken}] reward={ep.reward:.3f} done={ep.done} prompt='{prompt}' response='{resp}' "
                  f"info_keys={keys}")
            taken += 1
        remaining -= min(remaining, len(eb.episodes))
    if rewards:
        print(f"Collected {len(rewards)} episodes. reward_mean={float(np.mean(rewards)):.3f} "
              f"reward_std={float(np.std(rewards)):.3f}")
    else:
        print("No episodes collected.")
    return rewards


__all__ = ["PreparedPrompt", "Episode", "EpisodeBatch", "encode_images", "prepare_prompts", "collect_episodes",
           "episodes_to_training_batch", "main"]


if __name__ == "__main__":
    main()
