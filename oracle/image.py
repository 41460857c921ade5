"""numpy restatement of the reference's image preprocessing (test oracle only).

``preprocess_image_batch`` (crates/jammi-ai/src/inference/image_preprocess.rs:15-51):
each decoded image is padded to a white square (``pad_to_square``, :54-75,
centred at ((size - w) / 2, (size - h) / 2)), resized to ``target x target``
with ``FilterType::CatmullRom`` (``resize_exact``), and normalised per channel
as ``(pixel / 255 - mean) / std`` into a ``[B, 3, target, target]`` f32 tensor.

The resampling itself lives in the ``image`` crate, version 0.25.10 (the
reference's Cargo.lock), which is not vendored here.  Its published algorithm
is restated: a separable filter, vertical pass first into an f32 intermediate,
then horizontal with each result clamped to [0, 255] and rounded half away from
zero.  For output coordinate o of a pass with ratio r = src / dst:
centre c = (o + 0.5) r, support s = 2 max(r, 1), taps i in
[clamp(floor(c - s), 0, src - 1), clamp(ceil(c + s), left + 1, src)), weight
k((i - (c - 0.5)) / max(r, 1)) with k the Catmull-Rom cubic (the
Mitchell-Netravali BC-spline with B = 0, C = 1/2), weights divided by their
sum; each sum runs over the taps in order.  Every step is float32 with one
rounding per operation (no fused multiply-add), as the crate computes it, so
the restatement is exact to the bit wherever the operation order is.  Parity
against the crate itself is unpinned (no Rust toolchain here); the reference's
own known answers (image_preprocess.rs:95-146) pin the padding, the shapes and
the normalisation.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
OPENAI_CLIP_MEAN = (0.48145466, 0.4578275, 0.40821073)  # open_clip_vit.rs:15
OPENAI_CLIP_STD = (0.26862954, 0.26130258, 0.27577711)


def catmull_rom(x: np.float32) -> np.float32:
    """Mitchell-Netravali cubic with B = 0, C = 1/2 in float32, the polynomial
    evaluated left to right: k = ((A a^3 + B a^2) + C a + D) / 6."""
    a = F32(abs(F32(x)))
    a2 = F32(a * a)
    a3 = F32(a2 * a)
    if a < F32(1.0):
        k = F32(F32(F32(9.0) * a3) + F32(F32(-15.0) * a2))
        k = F32(k + F32(6.0))
    elif a < F32(2.0):
        k = F32(F32(F32(-3.0) * a3) + F32(F32(15.0) * a2))
        k = F32(k + F32(F32(-24.0) * a))
        k = F32(k + F32(12.0))
    else:
        k = F32(0.0)
    return F32(k / F32(6.0))


def taps(o: int, src: int, dst: int):
    """(left, normalised weights) of output coordinate o of one pass."""
    ratio = F32(F32(src) / F32(dst))
    sratio = ratio if ratio >= F32(1.0) else F32(1.0)
    support = F32(F32(2.0) * sratio)
    centre = F32(F32(F32(o) + F32(0.5)) * ratio)
    left = int(np.floor(F32(centre - support)))
    left = min(max(left, 0), src - 1)
    right = int(np.ceil(F32(centre + support)))
    right = min(max(right, left + 1), src)
    centre = F32(centre - F32(0.5))
    ws = [catmull_rom(F32(F32(F32(i) - centre) / sratio)) for i in range(left, right)]
    total = F32(0.0)
    for w in ws:
        total = F32(total + w)
    return left, [F32(w / total) for w in ws]


def pad_to_square(img: np.ndarray) -> np.ndarray:
    """``pad_to_square`` (image_preprocess.rs:54-75) of an RGB8 ``[h, w, 3]``."""
    h, w, _ = img.shape
    if w == h:
        return img
    size = max(w, h)
    canvas = np.full((size, size, 3), 255, dtype=np.uint8)
    y0, x0 = (size - h) // 2, (size - w) // 2
    canvas[y0:y0 + h, x0:x0 + w] = img
    return canvas


def resize_catmull_rom(img: np.ndarray, target: int) -> np.ndarray:
    """``resize_exact(target, target, CatmullRom)`` of a square RGB8 image ->
    RGB8 ``[target, target, 3]``."""
    src = img.shape[0]
    if src == target:
        return img.copy()
    v = img.astype(F32)
    inter = np.zeros((target, src, 3), dtype=F32)
    for oy in range(target):  # vertical pass, f32 intermediate
        left, ws = taps(oy, src, target)
        t = np.zeros((src, 3), dtype=F32)
        for i, w in enumerate(ws):
            t = t + v[left + i] * w
        inter[oy] = t
    out = np.zeros((target, target, 3), dtype=np.uint8)
    for ox in range(target):  # horizontal pass, clamp and round half away from zero
        left, ws = taps(ox, src, target)
        t = np.zeros((target, 3), dtype=F32)
        for i, w in enumerate(ws):
            t = t + inter[:, left + i] * w
        t = np.clip(t, F32(0.0), F32(255.0))
        fl = np.floor(t)
        out[:, ox] = np.where(t - fl >= F32(0.5), fl + F32(1.0), fl).astype(np.uint8)
    return out


def preprocess_image_batch(images, target: int, mean=OPENAI_CLIP_MEAN, std=OPENAI_CLIP_STD):
    """RGB8 images (any sizes) -> f32 ``[B, 3, target, target]``."""
    if not images:
        raise ValueError("Cannot preprocess empty image batch")
    m = np.asarray(mean, dtype=F32)
    s = np.asarray(std, dtype=F32)
    out = np.zeros((len(images), 3, target, target), dtype=F32)
    for b, img in enumerate(images):
        rgb = resize_catmull_rom(pad_to_square(np.asarray(img, dtype=np.uint8)), target)
        px = rgb.astype(F32) / F32(255.0)
        out[b] = ((px - m) / s).transpose(2, 0, 1)
    return out


def random_images(seed: int, sizes):
    """Seeded RGB8 test images: smooth gradients plus noise, [h, w, 3] each."""
    rng = np.random.default_rng(seed)
    out = []
    for (w, h) in sizes:
        yy, xx = np.mgrid[0:h, 0:w]
        base = np.stack([xx * 255.0 / max(w - 1, 1), yy * 255.0 / max(h - 1, 1),
                         (xx + yy) * 127.0 / max(w + h - 2, 1)], axis=-1)
        noise = rng.normal(0, 40, size=(h, w, 3))
        out.append(np.clip(base + noise, 0, 255).astype(np.uint8))
    return out
