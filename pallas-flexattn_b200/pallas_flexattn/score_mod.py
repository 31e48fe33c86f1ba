"""Score modification functions.

The reference advertises score_mod (README.md:8) but has none in code; this
module defines them with FlexAttention's contract: ``score_mod(score, b, h,
q_idx, kv_idx) -> score`` applied to the scaled logit before masking.  Each one
carries a ``ScoreSpec`` (attribute ``__fa_spec__``), its entry in the compiled
functor registry of libflexattn.  The registry applies, in this order: ALiBi,
relative bias, tanh softcap.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable, Optional

import torch

from . import _lib as L

ScoreMod = Callable[[Any, Any, Any, Any, Any], Any]


@dataclass(frozen=True, eq=False)
class ScoreSpec:
    flags: int = 0
    softcap: float = 0.0
    alibi_slopes: Optional[torch.Tensor] = None  # [H] fp32
    rel_bias: Optional[torch.Tensor] = None      # [H or 1, Tq + Tkv - 1] fp32
    _dev: dict = field(default_factory=dict, repr=False, compare=False)

    def key(self) -> tuple:
        return (self.flags, self.softcap, id(self.alibi_slopes), id(self.rel_bias))

    def device_tensors(self, device: torch.device) -> dict:
        k = str(device)
        if k not in self._dev:
            d = {}
            if self.alibi_slopes is not None:
                d["slopes"] = self.alibi_slopes.to(device=device, dtype=torch.float32).contiguous()
            if self.rel_bias is not None:
                d["bias"] = self.rel_bias.to(device=device, dtype=torch.float32).contiguous()
            self._dev[k] = d
        return self._dev[k]

    def to_c(self, device: torch.device, H: int, Tq: int, Tkv: int) -> L.FaScoreSpec:
        s = L.FaScoreSpec()
        s.flags = self.flags
        s.softcap = float(self.softcap)
        dev = self.device_tensors(device)
        if self.flags & L.FA_SCORE_ALIBI:
            if dev["slopes"].numel() != H:
                raise ValueError(f"ALiBi has {dev['slopes'].numel()} slopes for {H} heads")
            s.alibi_slopes = dev["slopes"].data_ptr()
        if self.flags & L.FA_SCORE_REL_BIAS:
            bias = dev["bias"]
            if bias.dim() != 2 or bias.shape[1] != Tq + Tkv - 1 or bias.shape[0] not in (1, H):
                raise ValueError(f"relative bias must be [1 or H, Tq+Tkv-1], got {tuple(bias.shape)}")
            s.rel_bias = bias.data_ptr()
            s.rel_bias_stride_h = bias.shape[1] if bias.shape[0] > 1 else 0
        return s


def spec_of(score_mod: Optional[ScoreMod]) -> Optional[ScoreSpec]:
    if score_mod is None:
        return ScoreSpec()
    return getattr(score_mod, "__fa_spec__", None)


def alibi_slopes(num_heads: int) -> torch.Tensor:
    """Standard ALiBi slopes ``2^(-8 h / H)`` for h = 1..H."""
    return torch.tensor([2.0 ** (-8.0 * h / num_heads) for h in range(1, num_heads + 1)], dtype=torch.float32)


def _idx(t, like):
    return t.to(like.device) if isinstance(t, torch.Tensor) and isinstance(like, torch.Tensor) else t


def alibi_score_mod(num_heads: Optional[int] = None, slopes=None) -> ScoreMod:
    """``score + slope[h] * (kv_idx - q_idx)``."""
    if slopes is None:
        if num_heads is None:
            raise ValueError("alibi_score_mod needs num_heads or slopes")
        slopes = alibi_slopes(num_heads)
    sl = torch.as_tensor(slopes, dtype=torch.float32)

    def score_mod(score, b, h, q_idx, kv_idx):
        s = _idx(sl, score)[h]
        return score + s * (kv_idx - q_idx)

    score_mod.__fa_spec__ = ScoreSpec(flags=L.FA_SCORE_ALIBI, alibi_slopes=sl)
    return score_mod


def softcap_score_mod(cap: float) -> ScoreMod:
    """``cap * tanh(score / cap)``."""
    cap = float(cap)
    if not cap > 0:
        raise ValueError("softcap must be positive")

    def score_mod(score, b, h, q_idx, kv_idx):
        return cap * torch.tanh(score / cap)

    score_mod.__fa_spec__ = ScoreSpec(flags=L.FA_SCORE_SOFTCAP, softcap=cap)
    return score_mod


def relative_bias_score_mod(bias) -> ScoreMod:
    """``score + bias[h, q_idx - kv_idx + Tkv - 1]`` for a [H or 1, Tq + Tkv - 1] table."""
    tb = torch.as_tensor(bias, dtype=torch.float32)
    if tb.dim() == 1:
        tb = tb[None]

    def score_mod(score, b, h, q_idx, kv_idx):
        t = _idx(tb, score)
        Tkv = score.shape[-1]
        hh = h if t.shape[0] > 1 else h * 0
        return score + t[hh, (q_idx - kv_idx + Tkv - 1)]

    score_mod.__fa_spec__ = ScoreSpec(flags=L.FA_SCORE_REL_BIAS, rel_bias=tb)
    return score_mod


def compose_score_mods(*mods: ScoreMod) -> ScoreMod:
    """Apply registry score_mods in the registry's order (ALiBi, relative bias, softcap)."""
    specs = [spec_of(m) for m in mods]
    if any(s is None for s in specs):
        raise NotImplementedError("compose_score_mods: every part needs a registry spec")
    order = {L.FA_SCORE_ALIBI: 0, L.FA_SCORE_REL_BIAS: 1, L.FA_SCORE_SOFTCAP: 2}
    pairs = sorted(zip(specs, mods), key=lambda p: order.get(p[0].flags, 3))
    flags, cap, slopes, bias = 0, 0.0, None, None
    for s, _ in pairs:
        if s.flags & flags:
            raise NotImplementedError("compose_score_mods: each kind at most once")
        flags |= s.flags
        cap = s.softcap or cap
        slopes = s.alibi_slopes if s.alibi_slopes is not None else slopes
        bias = s.rel_bias if s.rel_bias is not None else bias
    ordered = [m for _, m in pairs]

    def score_mod(score, b, h, q_idx, kv_idx):
        for m in ordered:
            score = m(score, b, h, q_idx, kv_idx)
        return score

    score_mod.__fa_spec__ = ScoreSpec(flags=flags, softcap=cap, alibi_slopes=slopes, rel_bias=bias)
    return score_mod



def slice_heads(score_mod: Optional[ScoreMod], h0: int, h1: int) -> Optional[ScoreMod]:
    """The same registry score_mod restricted to heads [h0, h1): per-head ALiBi slopes and
    relative-bias rows are sliced, head-independent parts are kept.  For head-sharded
    execution, where a rank runs heads h0..h1-1 of the full problem as its heads 0..h1-h0-1."""
    spec = spec_of(score_mod)
    if spec is None:
        raise NotImplementedError("slice_heads: the score_mod has no registry entry")
    if spec.flags == 0:
        return score_mod
    parts = []
    if spec.flags & L.FA_SCORE_ALIBI:
        parts.append(alibi_score_mod(slopes=spec.alibi_slopes[h0:h1]))
    if spec.flags & L.FA_SCORE_REL_BIAS:
        bias = spec.rel_bias if spec.rel_bias.shape[0] == 1 else spec.rel_bias[h0:h1]
        parts.append(relative_bias_score_mod(bias))
    if spec.flags & L.FA_SCORE_SOFTCAP:
        parts.append(softcap_score_mod(spec.softcap))
    return parts[0] if len(parts) == 1 else compose_score_mods(*parts)
