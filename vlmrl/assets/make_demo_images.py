"""Draw the caption environment's demo images (``vlmrl/assets/imgs/*.png``).

The captioning demo (``vlmrl.envs.vision_caption``) asks about seven scenes: a news banner about Nasdaq
futures, a fighter jet taking off, a traditional ceremony, a mountain landscape, a climbing panda, a
stadium seen from above and a desk with a laptop and coffee.  This script renders simple, deterministic
vector drawings of those scenes with PIL, so the environment runs offline on images that show what its
questions ask about.  Run ``python -m vlmrl.assets.make_demo_images`` to regenerate them.
"""

from __future__ import annotations

import math
from pathlib import Path

from PIL import Image, ImageDraw

SIZE = 448
OUT = Path(__file__).resolve().parent / "imgs"


def _sky(d: ImageDraw.ImageDraw, top, bottom, h=SIZE):
    for y in range(h):
        t = y / (h - 1)
        d.line([(0, y), (SIZE, y)], fill=tuple(int(a + (b - a) * t) for a, b in zip(top, bottom)))


def news() -> Image.Image:
    im = Image.new("RGB", (SIZE, SIZE), (18, 28, 60))
    d = ImageDraw.Draw(im)
    d.rectangle([0, 0, SIZE, 70], fill=(160, 10, 20))
    d.text((16, 22), "FOX BUSINESS NEWS  LIVE", fill=(255, 255, 255))
    d.rectangle([24, 100, SIZE - 24, 300], outline=(200, 200, 220), width=2)
    pts = [(24 + i * 20, 260 - int(60 * math.sin(i / 2.5)) - i * 4) for i in range(21)]
    d.line(pts, fill=(40, 220, 90), width=3)
    d.text((36, 110), "NASDAQ FUTURES  +1.2%", fill=(255, 255, 255))
    d.rectangle([0, SIZE - 90, SIZE, SIZE], fill=(240, 240, 240))
    d.text((16, SIZE - 70), "FUTURES TRADING: NASDAQ 18,412  DOW 39,850  S&P 5,210", fill=(10, 10, 10))
    return im


def jet() -> Image.Image:
    im = Image.new("RGB", (SIZE, SIZE))
    d = ImageDraw.Draw(im)
    _sky(d, (90, 150, 220), (200, 225, 245))
    d.rectangle([0, 330, SIZE, SIZE], fill=(70, 70, 75))
    for x in range(0, SIZE, 60):
        d.rectangle([x, 385, x + 30, 392], fill=(235, 235, 235))
    body = [(120, 300), (330, 220), (360, 214), (340, 232), (140, 312)]
    d.polygon(body, fill=(110, 118, 125))
    d.polygon([(220, 262), (280, 170), (300, 176), (260, 262)], fill=(95, 102, 110))   # wing
    d.polygon([(140, 305), (150, 265), (168, 268), (160, 305)], fill=(95, 102, 110))   # tail fin
    d.ellipse([300, 212, 330, 226], fill=(40, 50, 70))                                  # canopy
    d.polygon([(100, 300), (130, 296), (132, 314), (96, 322)], fill=(255, 150, 40))    # afterburner
    return im


def ceremony() -> Image.Image:
    im = Image.new("RGB", (SIZE, SIZE), (236, 224, 200))
    d = ImageDraw.Draw(im)
    d.rectangle([0, 300, SIZE, SIZE], fill=(150, 110, 70))                              # wooden floor
    d.rectangle([40, 60, 408, 90], fill=(170, 30, 30))                                  # torii beam
    d.rectangle([80, 90, 100, 300], fill=(170, 30, 30))
    d.rectangle([348, 90, 368, 300], fill=(170, 30, 30))
    for cx, robe in ((170, (250, 250, 250)), (280, (20, 20, 30))):                      # two figures in kimono
        d.ellipse([cx - 18, 150, cx + 18, 186], fill=(240, 210, 180))
        d.polygon([(cx - 40, 300), (cx - 22, 190), (cx + 22, 190), (cx + 40, 300)], fill=robe)
    d.ellipse([205, 250, 245, 270], fill=(200, 40, 40))                                 # sake cup
    return im


def mountains() -> Image.Image:
    im = Image.new("RGB", (SIZE, SIZE))
    d = ImageDraw.Draw(im)
    _sky(d, (120, 170, 230), (220, 235, 250))
    d.polygon([(0, 330), (130, 120), (250, 330)], fill=(90, 100, 120))
    d.polygon([(150, 330), (300, 80), (448, 330)], fill=(75, 85, 105))
    d.polygon([(270, 130), (300, 80), (330, 130), (310, 122), (300, 135), (288, 124)], fill=(250, 250, 255))
    d.polygon([(110, 150), (130, 120), (150, 150)], fill=(245, 245, 250))
    d.rectangle([0, 330, SIZE, SIZE], fill=(60, 120, 60))
    for x in range(10, SIZE, 34):                                                       # pine trees
        d.polygon([(x, 400), (x + 12, 350), (x + 24, 400)], fill=(30, 80, 40))
    return im


def panda() -> Image.Image:
    im = Image.new("RGB", (SIZE, SIZE), (140, 190, 120))
    d = ImageDraw.Draw(im)
    d.rectangle([200, 0, 240, SIZE], fill=(110, 80, 50))                                # tree trunk
    d.ellipse([150, 190, 290, 330], fill=(245, 245, 245))                               # body
    d.ellipse([160, 110, 260, 200], fill=(250, 250, 250))                               # head
    for ex in (168, 232):
        d.ellipse([ex - 12, 100, ex + 14, 126], fill=(20, 20, 20))                      # ears
    for ex in (190, 228):
        d.ellipse([ex - 12, 140, ex + 6, 162], fill=(20, 20, 20))                       # eye patches
    d.ellipse([203, 168, 217, 178], fill=(20, 20, 20))                                  # nose
    for arm in ([140, 200, 205, 235], [235, 215, 300, 250], [160, 300, 215, 335], [230, 290, 285, 325]):
        d.ellipse(arm, fill=(20, 20, 20))                                               # limbs gripping the trunk
    return im


def stadium() -> Image.Image:
    im = Image.new("RGB", (SIZE, SIZE), (90, 95, 100))
    d = ImageDraw.Draw(im)
    d.ellipse([24, 60, 424, 388], fill=(200, 200, 205))                                 # stands
    d.ellipse([64, 100, 384, 348], fill=(170, 60, 50))                                  # running track
    d.rectangle([124, 150, 324, 298], fill=(50, 150, 60))                               # pitch
    d.rectangle([124, 150, 324, 298], outline=(250, 250, 250), width=2)
    d.line([(224, 150), (224, 298)], fill=(250, 250, 250), width=2)
    d.ellipse([204, 204, 244, 244], outline=(250, 250, 250), width=2)
    for y in range(0, SIZE, 48):                                                        # roads around the venue
        d.line([(0, y), (20, y)], fill=(230, 230, 120), width=2)
    return im


def desk() -> Image.Image:
    im = Image.new("RGB", (SIZE, SIZE), (210, 200, 190))
    d = ImageDraw.Draw(im)
    d.rectangle([0, 240, SIZE, SIZE], fill=(150, 105, 65))                              # desk top
    d.polygon([(90, 330), (300, 330), (330, 380), (60, 380)], fill=(60, 60, 66))        # laptop base
    d.rectangle([100, 170, 290, 328], fill=(45, 45, 50))                                # screen lid
    d.rectangle([110, 180, 280, 318], fill=(70, 130, 200))                              # screen
    for y in range(195, 310, 14):
        d.line([(122, y), (260, y)], fill=(220, 235, 250), width=2)                     # text on screen
    d.ellipse([340, 300, 410, 320], fill=(240, 240, 240))                               # coffee cup rim
    d.rectangle([340, 310, 410, 370], fill=(240, 240, 240))
    d.ellipse([346, 302, 404, 318], fill=(90, 50, 25))                                  # coffee
    d.arc([400, 320, 430, 355], start=270, end=90, fill=(240, 240, 240), width=5)       # handle
    return im


SCENES = {
    "foxnews.png": news,
    "f35_takeoff.png": jet,
    "japanese_ceremony.png": ceremony,
    "mountain_landscape.png": mountains,
    "panda_climbing.png": panda,
    "stadium_aerial.png": stadium,
    "coffee_laptop.png": desk,
}


def main(out: Path = OUT) -> None:
    out.mkdir(parents=True, exist_ok=True)
    for name, draw in SCENES.items():
        draw().save(out / name, optimize=True)


if __name__ == "__main__":
    main()
