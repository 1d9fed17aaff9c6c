"""Cross-observation FFN token reuse and the motion-adaptive 2F/4F schedule.

Mirror of the reference's ``WAMInfer/approximation.py`` interface:

* ``TokenReuse(buckets)`` with ``capacities``, ``begin`` and ``commit`` -- run
  once per request: the float32 RGB change test that marks rows mandatory
  (numpy for host images as in the reference; ``wamffn_rgb_mandatory`` on the
  device for uint8 CUDA images, bit-identical) and the refresh count rounded
  up to a capacity bucket (reference ``:8-52``);
* ``select_tokens(state, features)`` -- the per-request row selection on the
  device (``wamffn_select_tokens``): fp32 relative L1 score against the
  committed first-layer features, mandatory rows first, stable descending
  top-``count``, ascending order, future rows appended (reference ``:55-67``);
* ``MotionRefinement`` -- which Euler updates run the Transformer
  (reference ``:70-84``).
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from waminfer_b200 import _lib


class TokenReuse:
    """Per-stream history of the last committed observation."""

    def __init__(self, buckets):
        self.buckets = tuple(sorted(set(buckets)))
        if not self.buckets or self.buckets[0] < 1:
            raise ValueError("Refresh capacities must be positive integers")
        self.reset()

    def reset(self):
        self.key = None
        self.image = None
        self.features = None
        self.cache = None

    def capacities(self, n):
        """Prepared refresh counts for n current rows: the buckets below n, then n."""
        return tuple(b for b in self.buckets if b < n) + (n,)

    @staticmethod
    def mandatory_rows(rgb, previous, h: int, w: int) -> np.ndarray:
        """True for every h x w patch whose mean float32 |RGB change| exceeds 5."""
        diff = np.subtract(rgb, previous, dtype=np.float32)
        np.abs(diff, out=diff)
        patches = diff.reshape(h, rgb.shape[0] // h, w, rgb.shape[1] // w, 3)
        return patches.mean(axis=(1, 3, 4)).reshape(-1) > 5.0

    @staticmethod
    def mandatory_rows_device(rgb: torch.Tensor, previous: torch.Tensor, h: int, w: int) -> torch.Tensor:
        """``mandatory_rows`` on the GPU for uint8 HWC images (``wamffn_rgb_mandatory``):
        integer sums of |change| per patch, one float32 division, ``> 5``."""
        if rgb.dtype != torch.uint8 or previous.dtype != torch.uint8 or rgb.shape != previous.shape:
            raise ValueError("device observations must be uint8 HWC images of one shape")
        if not (rgb.is_cuda and previous.device == rgb.device):
            raise ValueError("device observations must be on one CUDA device")
        if rgb.shape[0] % h or rgb.shape[1] % w:
            raise ValueError(f"a {tuple(rgb.shape)} observation does not split into {h}x{w} patches")
        rgb, previous = rgb.contiguous(), previous.contiguous()
        out = torch.empty(h * w, dtype=torch.uint8, device=rgb.device)
        with torch.cuda.device(rgb.device):
            _lib.check(_lib.lib().wamffn_rgb_mandatory(torch.cuda.current_stream(rgb.device).cuda_stream,
                                                       rgb.data_ptr(), previous.data_ptr(), rgb.shape[0],
                                                       rgb.shape[1], h, w, out.data_ptr()))
        return out.bool()

    def begin(self, image, inputs, prompt, patch):
        """Plans one request: returns (reuse dict, observation to commit on success).
        A uint8 CUDA tensor observation is tested on the device; anything else
        (PIL images, numpy arrays) on the host as in the reference."""
        latents = inputs["latents"]
        h, w = latents.shape[-2] // patch[1], latents.shape[-1] // patch[2]
        n = h * w
        on_device = isinstance(image, torch.Tensor) and image.is_cuda
        if on_device:
            if image.dtype != torch.uint8:
                raise ValueError("device observations must be uint8 HWC images")
            rgb = image.detach().clone()  # own the snapshot: callers recycle camera buffers
        else:
            rgb = np.array(image, copy=True)
        if rgb.ndim != 3 or rgb.shape[-1] != 3 or latents.shape[2] < 2:
            raise ValueError("Token reuse requires one HWC RGB observation and future video frames")
        key = (prompt, tuple(latents.shape), tuple(rgb.shape))
        if key != self.key:
            self.reset()
        if self.image is None:
            mandatory = np.ones(n, dtype=bool)
        elif on_device and (isinstance(self.image, torch.Tensor) or self.image.dtype == np.uint8):
            previous = self.image if isinstance(self.image, torch.Tensor) else torch.from_numpy(self.image)
            mandatory = self.mandatory_rows_device(rgb, previous.to(rgb.device), h, w)
        else:
            host = rgb.cpu().numpy() if on_device else rgb
            previous = self.image.cpu().numpy() if isinstance(self.image, torch.Tensor) else self.image
            mandatory = self.mandatory_rows(host, previous, h, w)
        required = int(mandatory.sum())
        required += math.ceil(0.25 * (n - required))
        count = next(b for b in self.capacities(n) if b >= required)
        reuse = dict(
            n=n,
            count=count,
            mandatory=torch.as_tensor(mandatory, device=latents.device),
            features=self.features if count < n else None,
            cache=self.cache if count < n else None,
        )
        return reuse, (key, rgb)

    def commit(self, observation, features, cache):
        """Publishes a finished request's history (copies: a later failed request
        must not be able to overwrite it)."""
        self.key, self.image = observation
        self.features, self.cache = features.clone(), cache.clone()


def select_rows(now: torch.Tensor, before: torch.Tensor, mandatory: torch.Tensor | None, count: int, seq: int,
                features_out: torch.Tensor | None = None) -> torch.Tensor:
    """Device row selection: int64 [count + seq - n] indices (see module doc)."""
    if now.dim() != 2 or before.shape != now.shape:
        raise ValueError("now/before must both be [n, d]")
    n, dim = now.shape
    if not (now.is_cuda and before.device == now.device):
        raise ValueError("select_rows runs on the GPU")
    if now.dtype != torch.bfloat16 or before.dtype != torch.bfloat16 or now.stride(1) != 1:
        raise ValueError("features must be bf16 with contiguous rows")
    before = before.contiguous()
    if mandatory is not None:
        mandatory = mandatory.to(device=now.device, dtype=torch.uint8).contiguous()
    indices = torch.empty(count + seq - n, dtype=torch.int64, device=now.device)
    args = _lib.SelectArgs(
        now=now.data_ptr(), now_stride=now.stride(0), before=before.data_ptr(),
        mandatory=None if mandatory is None else mandatory.data_ptr(), n=n, dim=dim, count=count, seq=seq,
        indices=indices.data_ptr(), features_out=None if features_out is None else features_out.data_ptr())
    with torch.cuda.device(now.device):
        _lib.check(_lib.lib().wamffn_select_tokens(torch.cuda.current_stream(now.device).cuda_stream,
                                                   ctypes.byref(args)))
    return indices


def select_tokens(state, features):
    """Records the current rows as ``token_features`` and, when fewer than n rows
    are refreshed, the gather list ``token_indices`` (reference
    ``WAMInfer/approximation.py:55-67``)."""
    reuse = state.extras["token_reuse"]
    n, count = reuse["n"], reuse["count"]
    current = features[:, :n]
    if count < n:
        out = torch.empty((1, n, features.shape[-1]), dtype=features.dtype, device=features.device)
        indices = select_rows(current[0], reuse["features"][0], reuse["mandatory"], count, features.shape[1],
                              features_out=out[0])
        state.extras["token_features"] = out
        state.extras["token_indices"] = indices
    else:
        state.extras["token_features"] = current.contiguous()


class MotionRefinement:
    """2F/4F: the Transformer runs at updates 0 and 3, plus 6 and 9 when the
    coarse action displacement after update 3 is at most `threshold` metres."""

    def __init__(self, metric, threshold, schedule):
        if metric is None or len(schedule) != 11:
            raise ValueError("adaptive_2f4f requires 10 Euler updates and a motion_metric returning metres")
        self.metric, self.threshold = metric, threshold
        self.nfe, self.amplitude, self.residual = 2, None, None

    def full(self, index):
        return index in (0, 3) or (self.nfe == 4 and index in (6, 9))

    def decide(self, actions):
        self.amplitude = float(self.metric(actions))
        if not math.isfinite(self.amplitude) or self.amplitude < 0:
            raise ValueError("motion_metric must return a finite nonnegative displacement in metres")
        self.nfe = 2 if self.amplitude > self.threshold else 4
