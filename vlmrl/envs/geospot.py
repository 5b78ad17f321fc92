"""Geospot: street-view geolocation with a hierarchical geodesic reward.

Behavioural counterpart of reference ``envs/geospot.py:33-811``:

* response parsing: ``key: value`` lines (keys City / Region|State|Province /
  Country / Latitude|Lat / Longitude|Lon, bullets and markdown emphasis
  tolerated, first occurrence wins), then a comma/semicolon/pipe-delimited
  fallback where trailing numeric pairs in range become coordinates and the
  remaining fields fill city, region, country in order (``:169-293``);
* ``reward = sum_f w_f exp(-d_f / tau_f) / sum_f w_f`` over the fields whose
  distance exists (``:430-511``); country/region/city distances compare
  *geocoded* truth against *geocoded* prediction, coords compare the ground
  truth against the parsed coordinates; an unparseable response scores 0;
* haversine with R = 6371 km; the default taus 2000/500/100/25 km;
* the curriculum (0/100/300/600/1000 episodes), where the coordinate weight of
  a stage is ``max(city, 0.5 * region)`` (``:741-752``).

Differences by design: the geocoder is pluggable and offline by default
(``StaticGeocoder``: a JSON cache plus explicit entries, never the network);
``OnlineGeocoder`` wraps geopy's Nominatim when geopy is installed.  The
dataset loader reads an OSV5M CSV + image folder that is already on disk.
"""

from __future__ import annotations

import json
import math
import os
import re
import unicodedata
from dataclasses import asdict, dataclass, field, replace
from pathlib import Path
from typing import Callable, Dict, List, Optional, Protocol, Sequence, Tuple

from vlmrl.envs.base import BaseEnv, BaseState, resolve_eos_id
from vlmrl.utils.vlm import decode_tokens

EARTH_RADIUS_KM = 6371.0


# --------------------------------------------------------------------------- types
@dataclass(frozen=True)
class Coords:
    lat: float
    lon: float

    def __post_init__(self):
        if not -90.0 <= self.lat <= 90.0:
            raise ValueError(f"Invalid latitude: {self.lat}")
        if not -180.0 <= self.lon <= 180.0:
            raise ValueError(f"Invalid longitude: {self.lon}")


@dataclass(frozen=True)
class Location:
    city: str
    region: str
    country: str
    coords: Coords


@dataclass(frozen=True)
class Sample:
    idx: int
    image_path: str
    truth: Location


@dataclass(frozen=True)
class ParsedResponse:
    city: Optional[str]
    region: Optional[str]
    country: Optional[str]
    coords: Optional[Coords]
    raw_text: str
    format_valid: bool


@dataclass(frozen=True)
class FieldWeights:
    country: float = 1.0
    region: float = 1.0
    city: float = 1.0
    coords: float = 1.0


@dataclass(frozen=True)
class RewardConfig:
    tau_country_km: float = 2000.0
    tau_region_km: float = 500.0
    tau_city_km: float = 100.0
    tau_coord_km: float = 25.0
    coord_tolerance_km: float = 25.0
    field_weights: FieldWeights = field(default_factory=FieldWeights)


@dataclass(frozen=True)
class CurriculumStage:
    name: str
    episode_threshold: int
    weight_country: float
    weight_region: float
    weight_city: float


@dataclass(frozen=True)
class RewardResult:
    reward: float
    d_country: Optional[float]
    d_region: Optional[float]
    d_city: Optional[float]
    d_coords: Optional[float]
    k_country: float
    k_region: float
    k_city: float
    k_coords: float
    active_weight_sum: float
    within_tolerance: bool


class Geocoder(Protocol):
    def __call__(self, query: str) -> Optional[Coords]: ...


PROMPT_TEMPLATE = (
    "Look at the image and guess the location.\n"
    "Respond with EXACTLY these 5 lines, no extra text:\n"
    "City: <city name>\n"
    "Region: <state or region>\n"
    "Country: <country name or ISO-2 code>\n"
    "Latitude: <number between -90 and 90>\n"
    "Longitude: <number between -180 and 180>\n"
)

KEY_ALIASES = {
    "city": "city", "country": "country", "region": "region", "state": "region", "province": "region",
    "latitude": "lat", "lat": "lat", "longitude": "lon", "lon": "lon",
}

DEFAULT_CURRICULUM = [
    CurriculumStage("country_coarse", 0, 1.0, 0.0, 0.0),
    CurriculumStage("country", 100, 0.5, 0.0, 0.0),
    CurriculumStage("region", 300, 0.3, 0.4, 0.0),
    CurriculumStage("city", 600, 0.2, 0.3, 0.3),
    CurriculumStage("full", 1000, 0.15, 0.25, 0.4),
]

# Coordinates-only configuration: the reward of the synthetic benchmark env.
COORDS_ONLY = RewardConfig(field_weights=FieldWeights(country=0.0, region=0.0, city=0.0, coords=1.0))


# --------------------------------------------------------------------------- parsing
_LINE = re.compile(r"^\s*(?:[-*+•]\s*)?(?P<key>[A-Za-z][A-Za-z0-9\s\-/_.]*?)\s*:\s*(?P<value>.+)$")
_NUMBER = re.compile(r"-?\d+(?:[.,]\d+)?")
_ENUM_PREFIX = re.compile(r"^\s*(?:[-*+•]|\d+(?:[.)]))\s*")
_LABEL_PREFIX = re.compile(r"^[A-Za-z][A-Za-z0-9\s\-/_.]*:\s*")


def _as_float(token: str) -> Optional[float]:
    try:
        return float(token.replace(",", "."))
    except ValueError:
        return None


def _clean_value(raw: str) -> str:
    v = raw.strip().strip("`\"' \t")
    v = re.sub(r"^[*_`]+", "", v)
    v = re.sub(r"[*_`]+$", "", v)
    return v.strip()


def _parse_key_values(text: str) -> Dict[str, object]:
    found: Dict[str, object] = {}
    for line in text.splitlines():
        m = _LINE.match(line)
        if m is None:
            continue
        key = re.sub(r"\s+", " ", m.group("key").strip().lower().strip("*_`\"' "))
        field_name = KEY_ALIASES.get(key)
        if field_name is None or field_name in found:
            continue
        value = _clean_value(m.group("value"))
        if field_name in ("lat", "lon"):
            num = _NUMBER.search(value)
            parsed = _as_float(num.group(0)) if num else None
            if parsed is not None:
                found[field_name] = parsed
        elif value:
            found[field_name] = value
    return found


def _parse_delimited(text: str) -> Dict[str, object]:
    if not text or not any(d in text for d in ",;|"):
        return {}
    pieces: List[str] = []
    for line in text.splitlines():
        line = _ENUM_PREFIX.sub("", line.strip()) if line.strip() else ""
        pieces += [seg.strip() for seg in re.split(r"[,|;]", line) if seg.strip()]
    if len(pieces) < 3:
        return {}
    pieces = [_LABEL_PREFIX.sub("", p).strip() for p in pieces]
    numeric = [i for i, p in enumerate(pieces) if re.fullmatch(r"-?\d+(?:[.,]\d+)?", p) and _as_float(p) is not None]
    out: Dict[str, object] = {}
    used = set()
    n = len(pieces)
    if len(numeric) >= 2 and numeric[-2:] == [n - 2, n - 1]:
        lat, lon = _as_float(pieces[n - 2]), _as_float(pieces[n - 1])
        if -90 <= lat <= 90 and -180 <= lon <= 180:
            out["lat"], out["lon"] = lat, lon
            used = {n - 2, n - 1}
    texts = [p for i, p in enumerate(pieces) if i not in used and p]
    for name, val in zip(("city", "region", "country"), texts):
        out[name] = val
    return out


def parse_response(text: str) -> ParsedResponse:
    if not text:
        return ParsedResponse(None, None, None, None, text, False)
    fields = _parse_key_values(text)
    sources = {"key_value"} if fields else set()
    for k, v in _parse_delimited(text).items():
        if k not in fields and v is not None:
            fields[k] = v
            sources.add("inline_delimited")
    coords = None
    if "lat" in fields and "lon" in fields:
        try:
            coords = Coords(lat=float(fields["lat"]), lon=float(fields["lon"]))
        except ValueError:
            coords = None
    return ParsedResponse(
        city=fields.get("city"), region=fields.get("region"), country=fields.get("country"), coords=coords,
        raw_text=text, format_valid=bool(sources) and len(fields) >= 2,
    )


# --------------------------------------------------------------------------- normalisation
def _lookup_country(raw: str):
    try:
        import pycountry  # type: ignore
    except ImportError:
        return None
    try:
        return pycountry.countries.lookup(raw)
    except (LookupError, AttributeError):
        return None


def normalize_country(s: Optional[str]) -> Optional[str]:
    if not s or not s.strip():
        return None
    raw = s.strip()
    if re.fullmatch(r"[A-Za-z]{2}", raw):
        return raw.upper()
    match = _lookup_country(raw)
    return str(match.alpha_2).upper() if match is not None and hasattr(match, "alpha_2") else None


_PREFIXES = re.compile(r"^(state of|province of|community of|autonomous community of|region of|county of|city of)\s+")


def normalize_text(s: Optional[str]) -> Optional[str]:
    if not s:
        return None
    x = unicodedata.normalize("NFKD", str(s)).encode("ascii", "ignore").decode("ascii").strip().lower()
    x = _PREFIXES.sub("", x)
    x = re.sub(r"\bst\.?\s+", "saint ", x)
    x = re.sub(r"\bsankt\s+", "saint ", x)
    x = re.sub(r"\s+", " ", x.replace("-", " "))
    return x or None


def normalize_location(loc: Location) -> Location:
    return Location(city=normalize_text(loc.city) or "", region=normalize_text(loc.region) or "",
                    country=normalize_country(loc.country) or loc.country.upper(), coords=loc.coords)


# --------------------------------------------------------------------------- reward
def haversine_km(c1: Coords, c2: Coords) -> float:
    p1, p2 = math.radians(c1.lat), math.radians(c2.lat)
    dp, dl = p2 - p1, math.radians(c2.lon - c1.lon)
    a = math.sin(dp / 2) ** 2 + math.cos(p1) * math.cos(p2) * math.sin(dl / 2) ** 2
    return EARTH_RADIUS_KM * 2.0 * math.atan2(math.sqrt(a), math.sqrt(1.0 - a))


def coord_kernel(distance_km: float, tau_km: float) -> float:
    return math.exp(-distance_km / tau_km)


def _join(parts: Sequence[Optional[str]]) -> Optional[str]:
    kept = [str(p).strip() for p in parts if p is not None and str(p).strip()]
    return ", ".join(kept) if kept else None


def _country_query(raw: Optional[str]) -> Optional[str]:
    if not raw or not raw.strip():
        return None
    raw = raw.strip()
    match = None
    if re.fullmatch(r"[A-Za-z]{2}", raw):
        try:
            import pycountry  # type: ignore

            match = pycountry.countries.get(alpha_2=raw.upper())
        except ImportError:
            match = None
    if match is None:
        match = _lookup_country(raw)
    if match is None:
        return raw
    for attr in ("common_name", "name", "official_name"):
        val = getattr(match, attr, None)
        if val:
            return str(val)
    return str(match)


def _geocode_hierarchy(geocoder: Geocoder, city: str, region: str, country: str):
    """Geocode (country, region, city) queries, each nested inside its parents."""
    cq = _country_query(country)
    c = geocoder(cq) if cq else None
    r = geocoder(_join([region, cq])) if region and _join([region, cq]) else None
    t = geocoder(_join([city, region or None, cq])) if city and _join([city, region or None, cq]) else None
    return c, r, t


def compute_reward(truth: Location, pred: ParsedResponse, config: RewardConfig, geocoder: Geocoder) -> RewardResult:
    tc, tr, tt = _geocode_hierarchy(geocoder, truth.city, truth.region, truth.country)
    pc, pr, pt = _geocode_hierarchy(geocoder, pred.city or "", pred.region or "", pred.country or "")

    def dist(a, b):
        return haversine_km(a, b) if a is not None and b is not None else None

    d = {
        "country": dist(tc, pc), "region": dist(tr, pr), "city": dist(tt, pt),
        "coords": haversine_km(truth.coords, pred.coords) if pred.coords is not None else None,
    }
    taus = {"country": config.tau_country_km, "region": config.tau_region_km,
            "city": config.tau_city_km, "coords": config.tau_coord_km}
    kern = {f: (coord_kernel(d[f], taus[f]) if d[f] is not None else 0.0) for f in d}
    w = {f: (getattr(config.field_weights, f) if d[f] is not None else 0.0) for f in d}
    total_w = sum(w.values())
    reward = sum(w[f] * kern[f] for f in d) / total_w if total_w > 0 else 0.0
    return RewardResult(
        reward=reward, d_country=d["country"], d_region=d["region"], d_city=d["city"], d_coords=d["coords"],
        k_country=kern["country"], k_region=kern["region"], k_city=kern["city"], k_coords=kern["coords"],
        active_weight_sum=total_w,
        within_tolerance=bool(d["coords"] is not None and d["coords"] <= config.coord_tolerance_km),
    )


# --------------------------------------------------------------------------- geocoders
class StaticGeocoder:
    """Offline geocoder: explicit entries plus an optional JSON cache {query: [lat, lon]}."""

    def __init__(self, entries: Optional[Dict[str, Tuple[float, float]]] = None, cache_path: Optional[str] = None):
        self.table: Dict[str, Coords] = {}
        if cache_path and os.path.exists(cache_path):
            try:
                with open(cache_path, "r", encoding="utf-8") as fh:
                    for k, v in json.load(fh).items():
                        try:
                            self.table[k] = Coords(float(v[0]), float(v[1]))
                        except (TypeError, ValueError, IndexError):
                            pass
            except (OSError, ValueError):
                pass
        for k, (lat, lon) in (entries or {}).items():
            self.table[k] = Coords(lat, lon)

    def __call__(self, query: str) -> Optional[Coords]:
        return self.table.get(query.strip()) if query else None


class OnlineGeocoder(StaticGeocoder):
    """Nominatim lookups (requires geopy and network) memoised into the JSON cache."""

    def __init__(self, cache_path: Optional[str] = None, user_agent: str = "vlmrl-geospot"):
        cache_path = cache_path or str(Path.home() / ".cache/huggingface/datasets/osv5m/geocode_cache.json")
        super().__init__(cache_path=cache_path)
        self.cache_path = cache_path
        from geopy.geocoders import Nominatim  # type: ignore

        self._client = Nominatim(user_agent=user_agent)

    def __call__(self, query: str) -> Optional[Coords]:
        q = (query or "").strip()
        if not q:
            return None
        if q in self.table:
            return self.table[q]
        try:
            res = self._client.geocode(q, exactly_one=True, addressdetails=False, language="en", timeout=2)
            if res is None:
                return None
            c = Coords(float(res.latitude), float(res.longitude))
        except Exception:
            return None
        self.table[q] = c
        try:
            os.makedirs(os.path.dirname(self.cache_path), exist_ok=True)
            with open(self.cache_path, "w", encoding="utf-8") as fh:
                json.dump({k: [v.lat, v.lon] for k, v in self.table.items()}, fh)
        except OSError:
            pass
        return c


CachedGeocoder = OnlineGeocoder


def load_dataset(split: str = "test", root: Optional[str] = None, max_samples: int = -1) -> List[Sample]:
    """Read an on-disk OSV5M split: ``<root>/<split>.csv`` and ``<root>/images/<split>/<xx>/<id>.jpg``."""
    import pandas as pd

    base = Path(root) if root else Path.home() / ".cache/huggingface/datasets/osv5m"
    table = base / f"{split}.csv"
    if not table.exists():
        raise FileNotFoundError(f"OSV5M metadata not found at {table} (no network download in this framework)")
    df = pd.read_csv(table, dtype={"id": str})
    images = base / "images" / split
    out: List[Sample] = []
    for _, row in df.head(100000).iterrows():
        img_id = str(row["id"])
        folder = "00" if split == "test" else (img_id[:2] if len(img_id) >= 2 else "00")
        path = images / folder / f"{img_id}.jpg"
        if not path.exists():
            continue
        try:
            truth = Location(
                city=str(row["city"]) if pd.notna(row["city"]) else "",
                region=str(row["region"]) if pd.notna(row["region"]) else "",
                country=str(row["country"]) if pd.notna(row["country"]) else "",
                coords=Coords(float(row["latitude"]), float(row["longitude"])),
            )
        except (ValueError, KeyError):
            continue
        out.append(Sample(idx=len(out), image_path=str(path), truth=truth))
        if 0 < max_samples <= len(out):
            break
    if not out:
        raise ValueError(f"No valid samples found for OSV5M {split} dataset")
    return out


# --------------------------------------------------------------------------- env
@dataclass(frozen=True)
class OSV5MPrompt:
    question: str
    image: object
    image_path: str
    sample: Sample
    stage: CurriculumStage


@dataclass(frozen=True)
class OSV5MState(BaseState):
    sample: Sample
    image: object
    stage: CurriculumStage

    def render(self) -> str:
        return "Looking at this street view image, predict the location."


def stage_reward_config(base: RewardConfig, stage: CurriculumStage) -> RewardConfig:
    weights = FieldWeights(country=stage.weight_country, region=stage.weight_region, city=stage.weight_city,
                           coords=max(stage.weight_city, 0.5 * stage.weight_region))
    return replace(base, field_weights=weights)


def reward_info(text: str, parsed: ParsedResponse, truth: Location, cfg: RewardConfig,
                result: RewardResult, n_tokens: int, stage: CurriculumStage) -> Dict[str, object]:
    return {
        "response": text, "response_len_chars": len(text), "response_len_tokens": n_tokens,
        "stage": stage.name,
        "stage_weights": {"country": stage.weight_country, "region": stage.weight_region,
                          "city": stage.weight_city, "coords": cfg.field_weights.coords},
        "reward_field_weights": asdict(cfg.field_weights),
        "kernel_taus": {"country": cfg.tau_country_km, "region": cfg.tau_region_km,
                        "city": cfg.tau_city_km, "coords": cfg.tau_coord_km},
        "parsed": {"city": parsed.city, "region": parsed.region, "country": parsed.country,
                   "coords": [parsed.coords.lat, parsed.coords.lon] if parsed.coords else None,
                   "format_valid": parsed.format_valid},
        "ground_truth": {"city": truth.city, "region": truth.region, "country": truth.country,
                         "coords": [truth.coords.lat, truth.coords.lon]},
        **asdict(result),
    }


class GeospotEnv(BaseEnv):
    def __init__(self, tokenizer, split: str = "test", reward_config: Optional[RewardConfig] = None,
                 curriculum: Optional[List[CurriculumStage]] = None, geocoder: Optional[Callable] = None,
                 samples: Optional[List[Sample]] = None, data_root: Optional[str] = None,
                 max_samples: int = -1):
        super().__init__()
        self.tokenizer = tokenizer
        self.eos_token_id = resolve_eos_id(tokenizer)
        self.tokens_per_action = 256
        self.samples = samples if samples is not None else load_dataset(split, data_root, max_samples)
        self.num_tasks = len(self.samples)
        self._base_reward_config = reward_config or RewardConfig()
        self.reward_config = self._base_reward_config
        self.curriculum = sorted(curriculum or DEFAULT_CURRICULUM, key=lambda s: s.episode_threshold)
        self.geocoder = geocoder if geocoder is not None else StaticGeocoder()
        self.episode_count = 0

    def _current_stage(self) -> CurriculumStage:
        active = self.curriculum[0]
        for stage in self.curriculum:
            if self.episode_count >= stage.episode_threshold:
                active = stage
        return active

    def _config_for_stage(self, stage: CurriculumStage) -> RewardConfig:
        return stage_reward_config(self._base_reward_config, stage)

    def _load_image(self, sample: Sample):
        from PIL import Image

        return Image.open(sample.image_path).convert("RGB")

    def reset(self, idx: int):
        sample = self.samples[idx % len(self.samples)]
        image = self._load_image(sample)
        stage = self._current_stage()
        self.episode_count += 1
        return (OSV5MState(sample=sample, image=image, stage=stage),
                OSV5MPrompt(question=PROMPT_TEMPLATE, image=image, image_path=sample.image_path,
                            sample=sample, stage=stage))

    def step(self, state: OSV5MState, action_tokens):
        if self.eos_token_id is not None:
            action_tokens = self.clean_action(action_tokens, self.eos_token_id)
        text = decode_tokens(self.tokenizer, action_tokens).strip()
        parsed = parse_response(text)
        cfg = self._config_for_stage(state.stage)
        result = compute_reward(state.sample.truth, parsed, cfg, self.geocoder)
        info = reward_info(text, parsed, state.sample.truth, cfg, result, len(action_tokens), state.stage)
        return state, [], float(result.reward), True, info


__all__ = [
    "Coords", "Location", "Sample", "ParsedResponse", "FieldWeights", "RewardConfig", "CurriculumStage",
    "RewardResult", "PROMPT_TEMPLATE", "KEY_ALIASES", "DEFAULT_CURRICULUM", "COORDS_ONLY", "parse_response",
    "normalize_country", "normalize_text", "normalize_location", "haversine_km", "coord_kernel",
    "compute_reward", "StaticGeocoder", "OnlineGeocoder", "CachedGeocoder", "load_dataset", "GeospotEnv",
    "OSV5MPrompt", "OSV5MState", "stage_reward_config",
]
