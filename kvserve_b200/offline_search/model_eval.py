"""Accuracy of a compression profile measured through a language model's
own forward pass (role of
kvserve_v1/offline_search/evaluation/param_search/acc_evaluator.py:68-268).

The reference runs lm-eval tasks twice, once with the model's default cache
and once with a cache that stores the compressed-then-restored prefill KV,
and reports ``mean(custom_score / default_score) * 100``.  Datasets and
pretrained checkpoints need a network here, so the tasks are measured on
the model's own greedy continuations, with the same normalisation:

* ``top1_agreement`` — the prompt is prefilled through
  :func:`~kvserve_b200.offline_search.cache_sim.simulated_cache` (the prefill
  KV is replaced by the profile's reconstruction), then the default run's
  greedy continuation is fed back one token at a time (decode tokens stay
  uncompressed, as in the reference's custom cache); the score is the share
  of steps whose argmax equals the default run's.  Default score: 1.
* ``continuation_likelihood`` — ``exp`` of the mean log-probability that the
  degraded run assigns to the default continuation minus the default run's
  own mean log-probability (1 when nothing changed, lower when the KV error
  moves probability mass away).  Default score: 1.

Any Hugging Face causal LM works (``from_pretrained`` of a local checkpoint
with real prompts gives the reference's setting minus the task datasets);
:func:`tiny_llama` builds a random-init Llama for tests and the CLI.  An
lm-eval-style scorer plugs in as ``task_scores(model, make_cache) ->
{task: score}``; the evaluator then normalises its scores the same way.

    python -m kvserve_b200.offline_search.model_eval \
        configs/compression/hadamard_k4v2_bitpack.json [more profiles...]
"""
from __future__ import annotations

import argparse
import json
import math
from typing import Callable, Optional, Sequence

import torch

from .cache_sim import KVServeSim, simulated_cache

TaskScorer = Callable[[torch.nn.Module, Callable[[], object]], dict]


def tiny_llama(layers: int = 4, hidden: int = 256, heads: int = 4, kv_heads: int = 2, vocab: int = 512,
               init_std: float = 0.02, seed: int = 0) -> torch.nn.Module:
    """A random-init Llama (head_dim = hidden / heads, the standard 0.02
    initialisation), fp32 on the CPU."""
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(vocab_size=vocab, hidden_size=hidden, intermediate_size=2 * hidden, num_hidden_layers=layers,
                      num_attention_heads=heads, num_key_value_heads=kv_heads, max_position_embeddings=4096,
                      initializer_range=init_std, attn_implementation="eager")
    return LlamaForCausalLM(cfg).eval()


def _kv_geometry(model: torch.nn.Module) -> tuple[int, int, int]:
    c = model.config
    head_dim = getattr(c, "head_dim", None) or c.hidden_size // c.num_attention_heads
    return c.num_hidden_layers, c.num_key_value_heads, head_dim


class ModelAccuracyEvaluator:
    """``evaluate(profile) -> score`` in percent of the default cache's
    scores (100 = indistinguishable), averaged over tasks."""

    def __init__(self, model: torch.nn.Module, prompts: Sequence[torch.Tensor], new_tokens: int = 16,
                 task_scores: Optional[TaskScorer] = None):
        self.model = model
        self.prompts = [p.reshape(1, -1).long() for p in prompts]
        self.new_tokens = new_tokens
        self.L, self.H, self.D = _kv_geometry(model)
        self.task_scores = task_scores
        self.last: dict = {}
        # the default run: greedy continuation and its per-step log-probabilities
        self._ref = [self._rollout(p, None) for p in self.prompts]
        self.default_scores = (task_scores(model, self._default_cache) if task_scores else None)

    def _default_cache(self):
        from transformers import DynamicCache
        return DynamicCache()

    @torch.no_grad()
    def _rollout(self, prompt: torch.Tensor, forced: Optional[torch.Tensor], cache=None):
        """Prefill ``prompt`` into ``cache`` and run ``new_tokens`` decode
        steps, feeding ``forced`` (teacher forcing) or the argmax.  Returns
        (tokens, argmaxes, log-probabilities of the fed tokens)."""
        if cache is None:
            cache = self._default_cache()
        out = self.model(input_ids=prompt, past_key_values=cache, use_cache=True)
        logits = out.logits[:, -1].float()
        toks, tops, lps = [], [], []
        for i in range(self.new_tokens):
            top = int(logits.argmax(-1))
            tok = top if forced is None else int(forced[i])
            tops.append(top)
            toks.append(tok)
            lps.append(float(torch.log_softmax(logits, -1)[0, tok]))
            if i + 1 == self.new_tokens:
                break
            out = self.model(input_ids=torch.tensor([[tok]]), past_key_values=out.past_key_values, use_cache=True)
            logits = out.logits[:, -1].float()
        return torch.tensor(toks), torch.tensor(tops), torch.tensor(lps)

    def make_cache(self, profile: dict):
        sim = KVServeSim(profile, self.H, self.D, num_layers=self.L)

        def bf16_sim(kv):
            # the served KV is bf16: compress that, hand the model its dtype back
            rec, ratio = sim(kv.to(torch.bfloat16))
            return rec.to(kv.dtype), ratio
        return lambda: simulated_cache(bf16_sim, self.L)

    def sim_cache(self, sim):
        """Caches that apply any simulator of :mod:`.cache_sim` (KIVI,
        CacheGen, ...) to the bf16 prefill KV, like :meth:`make_cache` does
        for a profile."""
        def bf16_sim(kv):
            rec, ratio = sim(kv.to(torch.bfloat16))
            return rec.to(kv.dtype), ratio
        return lambda: simulated_cache(bf16_sim, self.L)

    def task_breakdown(self, profile: dict) -> dict:
        return self._breakdown(self.make_cache(profile))

    def _breakdown(self, make) -> dict:
        agree, like, ratios = [], [], []
        for p, (toks, _, lps) in zip(self.prompts, self._ref):
            cache = make()
            _, tops, lps_c = self._rollout(p, toks, cache)
            agree.append(float((tops == toks).float().mean()))
            like.append(math.exp(float(lps_c.mean() - lps.mean())))
            ratios += list(cache.ratios.values())
        scores = {"top1_agreement": sum(agree) / len(agree),
                  "continuation_likelihood": min(1.0, sum(like) / len(like))}
        defaults = {"top1_agreement": 1.0, "continuation_likelihood": 1.0}
        if self.task_scores is not None:
            scores.update(self.task_scores(self.model, make))
            defaults.update(self.default_scores)
        return {"scores": scores, "defaults": defaults,
                "compression_ratio": (sum(ratios) / len(ratios)) if ratios else 1.0}

    def evaluate(self, profile: dict) -> float:
        return self._score(self.task_breakdown(profile))

    def evaluate_sim(self, sim) -> float:
        """The same score for a baseline method's simulator (the reference's
        method comparison, e.g. scripts/run_hotpotqa_4way.sh, on these tasks)."""
        return self._score(self._breakdown(self.sim_cache(sim)))

    def _score(self, b: dict) -> float:
        rel = [b["scores"][k] / b["defaults"][k] for k in b["scores"] if b["defaults"].get(k)]
        self.last = dict(b, avg_score=round(100.0 * sum(rel) / len(rel), 2))
        return self.last["avg_score"]


@torch.no_grad()
def capture_kv(model: torch.nn.Module, prompts: Sequence[torch.Tensor], dtype=torch.bfloat16) -> torch.Tensor:
    """The prefill KV a causal LM produces for ``prompts`` (equal lengths), as
    the ``[L, 2, B, S, H, D]`` sample the offline search and the evaluators
    take (role of the reference's KV fixture capture,
    scripts/capture_kv_fixture.py)."""
    from transformers import DynamicCache
    ids = torch.stack([p.reshape(-1).long() for p in prompts])
    cache = DynamicCache()
    model(input_ids=ids, past_key_values=cache, use_cache=True)
    layers = []
    for layer in cache.layers:
        k, v = layer.keys, layer.values                 # [B, H, S, D]
        layers.append(torch.stack([k, v]).permute(0, 1, 3, 2, 4))
    return torch.stack(layers).to(dtype)


def synthetic_prompts(count: int, length: int, vocab: int, seed: int = 0) -> list[torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (length,), generator=g) for _ in range(count)]


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("profiles", nargs="*", help="compression profile JSON files")
    ap.add_argument("--baselines", default="",
                    help="comma-separated baseline methods to score too: kivi2, kivi4, cachegen")
    ap.add_argument("--model", default=None, help="local Hugging Face checkpoint (default: random-init tiny Llama)")
    ap.add_argument("--prompts", type=int, default=4)
    ap.add_argument("--prompt-len", type=int, default=256)
    ap.add_argument("--new-tokens", type=int, default=16)
    ap.add_argument("--capture", default=None,
                    help="also save the prompts' prefill KV [L, 2, B, S, H, D] here (for search --kv)")
    args = ap.parse_args()
    if args.model:
        from transformers import AutoModelForCausalLM
        model = AutoModelForCausalLM.from_pretrained(args.model, torch_dtype=torch.float32).eval()
    else:
        model = tiny_llama()
    prompts = synthetic_prompts(args.prompts, args.prompt_len, model.config.vocab_size)
    if args.capture:
        torch.save(capture_kv(model, prompts), args.capture)
    ev = ModelAccuracyEvaluator(model, prompts, new_tokens=args.new_tokens)
    for path in args.profiles:
        with open(path) as f:
            prof = json.load(f)
        score = ev.evaluate(prof)
        print(json.dumps({"profile": path, "avg_score": score, "scores": ev.last["scores"],
                          "compression_ratio": round(ev.last["compression_ratio"], 3)}))
    from .cache_sim import CacheGenSim, KIVISim
    methods = {"kivi2": lambda: KIVISim(bits=2), "kivi4": lambda: KIVISim(bits=4), "cachegen": CacheGenSim}
    for name in filter(None, (x.strip() for x in args.baselines.split(","))):
        score = ev.evaluate_sim(methods[name]())
        print(json.dumps({"method": name, "avg_score": score, "scores": ev.last["scores"],
                          "compression_ratio": round(ev.last["compression_ratio"], 3)}))


if __name__ == "__main__":
    main()
