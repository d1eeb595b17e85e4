"""Host-side construction of a varlen prefill batch (CPU): the array version matches a
per-token loop over positions and KV-cache slots."""
import random

from swarm_inference_lab_b200.engine.kv_cache import PAGE
from swarm_inference_lab_b200.engine.runner import prefill_host_batch


def _loop(ids, starts, pages):
    flat, pos, slots, cu, seq_lens = [], [], [], [0], []
    for i in range(len(ids)):
        n = len(ids[i])
        flat.extend(ids[i])
        p = list(range(starts[i], starts[i] + n))
        pos.extend(p)
        slots.extend(pages[i][q // PAGE] * PAGE + q % PAGE for q in p)
        cu.append(cu[-1] + n)
        seq_lens.append(starts[i] + n)
    return flat, pos, slots, cu, seq_lens


def test_prefill_host_batch_matches_loop():
    rng = random.Random(0)
    for _ in range(20):
        B = rng.randint(1, 6)
        lens = [rng.randint(1, 300) for _ in range(B)]
        starts = [rng.randint(0, 200) for _ in range(B)]
        pages = [rng.sample(range(1000), (s + n + PAGE - 1) // PAGE) for s, n in zip(starts, lens)]
        ids = [[rng.randrange(50000) for _ in range(n)] for n in lens]
        h = prefill_host_batch(ids, starts, pages, max(len(p) for p in pages))
        flat, pos, slots, cu, seq_lens = _loop(ids, starts, pages)
        assert h["ids"].tolist() == flat and h["positions"].tolist() == pos
        assert h["slots"].tolist() == slots and h["cu"].tolist() == cu
        assert h["seq_lens"].tolist() == seq_lens and h["max_q_len"] == max(lens)
        for i, pg in enumerate(pages):
            assert h["block_table"][i, :len(pg)].tolist() == pg
