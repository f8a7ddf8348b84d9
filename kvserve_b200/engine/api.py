"""A vLLM-style entry point of the standalone PD engine.

    from kvserve_b200 import LLM
    llm = LLM("llama-3.1-8b", profile="k4v2", max_prompt=8192, max_new_tokens=128)
    outs = llm.generate([[1, 2, 3, ...], ...], max_tokens=64)
    llm.close()

One process per GPU under ``torchrun`` (a single process runs prefill and
decode colocated on one GPU); every rank calls :meth:`LLM.generate` with the
same prompts, as with any collective.  The ranks that hold the decoded tokens
(decode ranks, or the colocated process) get :class:`Output` objects with
tokens; the others get outputs with ``token_ids=None`` and the timings of
their side.  ``profile`` is a transfer profile of the KV hand-off: a name
(``k8v8``, ``k4v4``, ``k4v2``, ``k2v2``, ``off``/``raw``), a compression
profile dict or JSON file in the connector's configuration language
(``configs/compression/*.json``), or a
:class:`~kvserve_b200.engine.transfer.TransferProfile`.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import Any, Optional, Sequence

import torch


@dataclass
class Output:
    """One request's result: generated token ids (None on ranks that do not
    hold them) and its timings in ms (TTFT, hand-off, decode)."""
    prompt_len: int
    token_ids: Optional[list]
    timing: Any


def resolve_profile(profile: Any):
    """A :class:`TransferProfile` from a name, a compression profile (dict or
    JSON path) or a profile object."""
    from .serving import ENGINE_PROFILES
    from .transfer import TransferProfile
    if isinstance(profile, TransferProfile):
        return profile
    if profile is None or profile in ("raw", "off"):
        return TransferProfile.raw()
    if isinstance(profile, str) and profile in ENGINE_PROFILES:
        return ENGINE_PROFILES[profile]
    if isinstance(profile, str) and os.path.exists(profile):
        with open(profile) as f:
            return TransferProfile.from_compression(json.load(f))
    if isinstance(profile, (dict, str)):
        return TransferProfile.from_compression(profile)
    raise ValueError(f"unknown transfer profile {profile!r}")


class LLM:
    def __init__(self, model: str = "llama-3.1-8b", profile: Any = "k4v2", max_prompt: int = 8192,
                 max_new_tokens: int = 128, backend: str = "nccl", **engine_kwargs):
        from ..models.config import get_config
        from ..parallel.context import ParallelContext, init_parallel
        from .pd import PDEngine
        self.cfg = get_config(model)
        self.profile = resolve_profile(profile)
        distributed = int(os.environ.get("WORLD_SIZE", "1")) > 1
        self.ctx = init_parallel(backend) if distributed else ParallelContext()
        self.engine = PDEngine(self.cfg, self.ctx, self.profile, max_prompt=max_prompt,
                               max_new_tokens=max_new_tokens, **engine_kwargs)

    @property
    def holds_tokens(self) -> bool:
        """Whether this rank receives the generated tokens."""
        return self.ctx.is_decode

    def generate(self, prompts: Sequence[Any], max_tokens: Optional[int] = None) -> list[Output]:
        """Serve ``prompts`` (token-id lists or int tensors) one after the
        other; every rank must pass the same prompts."""
        outs = []
        for p in prompts:
            ids = p if isinstance(p, torch.Tensor) else torch.tensor(list(p), dtype=torch.int32)
            ids = ids.to(torch.int32).reshape(-1)
            if torch.cuda.is_available():
                ids = ids.pin_memory()
            res = self.engine.generate(ids, max_tokens)
            outs.append(Output(int(ids.numel()), res.tokens if self.holds_tokens else None, res.timing))
        return outs

    def close(self) -> None:
        from ..parallel.context import destroy_parallel
        self.engine.close()
        if self.ctx.distributed:
            destroy_parallel(self.ctx)
