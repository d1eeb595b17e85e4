"""Exact speculative decoding with prompt-lookup drafts and greedy verification.

Drafts come from the sequence itself: the most recent earlier occurrence of the
last ``ngram`` tokens proposes the ``k`` tokens that followed it (no draft model).
One verification pass runs ``[current token] + draft`` as a short causal chunk at
the end of the context (the paged prefill path), takes the greedy token of every
row, accepts the longest draft prefix that matches, and emits the accepted tokens
plus the verifier's next token.  The output is exactly the verifier's own greedy
continuation; KV rows written for rejected drafts lie beyond the accepted length
and are overwritten by the next chunk.

``SpeculativeDecoder`` drives one sequence through an ``LLMEngine``'s runner and
cache; ``max_draft=0`` degenerates to plain greedy decoding on the same path.
Drafting is disabled automatically for a sequence whose acceptance rate stays
below ``min_accept`` (a draft that is always rejected costs a wider verify pass).

Reference: prompt-lookup drafting and greedy verification of
si/experiments/experiment_011/drafting.py:10-82 (experiment only there; the product
stage runtime rejects VERIFY_CANDIDATES, si/worker/stage_runtime.py:2070-2071).
"""
from __future__ import annotations

from dataclasses import dataclass


def prompt_lookup_draft(tokens: list[int], k: int, ngram: int = 3, min_ngram: int = 1) -> list[int]:
    """Tokens that followed the latest earlier match of the context's trailing n-gram."""
    if k <= 0:
        return []
    for n in range(min(ngram, len(tokens) - 1), min_ngram - 1, -1):
        tail = tokens[-n:]
        for i in range(len(tokens) - n - 1, -1, -1):
            if tokens[i:i + n] == tail:
                follow = tokens[i + n:i + n + k]
                if follow:
                    return follow
    return []


@dataclass
class SpecStats:
    steps: int = 0
    drafted: int = 0
    accepted: int = 0
    emitted: int = 0

    @property
    def acceptance(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0

    @property
    def tokens_per_step(self) -> float:
        return self.emitted / self.steps if self.steps else 0.0


class SpeculativeDecoder:
    def __init__(self, engine, *, max_draft: int = 4, ngram: int = 3, min_accept: float = 0.1,
                 warmup_steps: int = 8):
        self.eng = engine
        self.k = max_draft
        self.ngram = ngram
        self.min_accept = min_accept
        self.warmup = warmup_steps

    def generate(self, prompt: list[int], max_new_tokens: int, seq_id: str = "spec") -> tuple[list[int], SpecStats]:
        eng = self.eng
        kv, runner = eng.kv, eng.runner
        st = SpecStats()
        kv.open(seq_id)
        try:
            kv.reserve(seq_id, len(prompt) + max_new_tokens + self.k + 1)
            pages = kv.seqs[seq_id].pages
            cur = int(runner.prefill([list(prompt)], [0], [pages])[0])
            out = [cur]
            ctx = len(prompt)              # positions with valid KV
            use_draft = self.k > 0
            while len(out) < max_new_tokens:
                draft = prompt_lookup_draft(list(prompt) + out, min(self.k, max_new_tokens - len(out) - 1),
                                            self.ngram) if use_draft else []
                g = runner.prefill([[cur] + draft], [ctx], [pages], all_rows=True).tolist()
                i = 0
                while i < len(draft) and draft[i] == g[i]:
                    i += 1
                new = g[: i + 1]
                st.steps += 1
                st.drafted += len(draft)
                st.accepted += i
                st.emitted += len(new)
                out.extend(new)
                ctx += i + 1
                cur = out[-1]
                if use_draft and st.steps >= self.warmup and st.acceptance < self.min_accept:
                    use_draft = False
            kv.seqs[seq_id].length = ctx
            return out[:max_new_tokens], st
        finally:
            kv.close(seq_id)
