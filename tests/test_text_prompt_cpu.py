"""Text prompts through the coordinator (CPU): a deployed Hugging Face checkpoint that carries
a tokenizer is asked with text; the coordinator tokenizes with the checkpoint's tokenizer, the
greedy tokens equal transformers' ``generate`` on the same ids, and the ``completed`` event
carries the decoded text.  A model without a tokenizer refuses a text prompt."""
import asyncio

import pytest
import torch

WORDS = [f"w{i}" for i in range(200)]


def _checkpoint(path):
    transformers = pytest.importorskip("transformers")
    from tokenizers import Tokenizer, models, pre_tokenizers
    vocab = {"[UNK]": 0, "[BOS]": 1, "[EOS]": 2}
    for w in WORDS:
        vocab[w] = len(vocab)
    tok = Tokenizer(models.WordLevel(vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    fast = transformers.PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="[UNK]",
                                                bos_token="[BOS]", eos_token="[EOS]")
    torch.manual_seed(0)
    hf = transformers.Qwen3ForCausalLM(transformers.Qwen3Config(
        vocab_size=256, hidden_size=64, intermediate_size=96, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=16, initializer_range=0.2,
        max_position_embeddings=256, tie_word_embeddings=False)).eval()
    hf.save_pretrained(path, safe_serialization=True)
    fast.save_pretrained(path)
    return hf, fast


def test_text_prompt_is_tokenized_by_the_coordinator(tmp_path):
    from swarm_inference_lab_b200.coordinator.service import CoordinatorCore, CoordinatorRpcServer
    from swarm_inference_lab_b200.runtime.worker_runtime import WorkerRuntime
    from swarm_inference_lab_b200.security.identity import Identity

    torch.set_num_threads(2)
    hf, fast = _checkpoint(tmp_path / "ck")
    text = "w5 w77 w100 w12 w199 w41 w8"
    ids = fast.encode(text)
    with torch.no_grad():
        want = hf.generate(torch.tensor([ids]), max_new_tokens=6, do_sample=False)[0, len(ids):].tolist()

    async def go():
        ident = Identity.generate("coordinator")
        core = CoordinatorCore(ident, require_member=False, heartbeat_timeout_s=30.0)
        rpc = CoordinatorRpcServer(core, host="127.0.0.1", port=0)
        port = await rpc.start()
        ws = []
        try:
            for i in range(2):
                w = WorkerRuntime(f"w{i}", Identity.generate(f"w{i}"), f"127.0.0.1:{port}",
                                  coordinator_fingerprint=ident.fingerprint, heartbeat_s=1.0,
                                  device="cpu")
                await w.start()
                ws.append(w)
            dep = await core.deploy({"model": {"checkpoint": str(tmp_path / "ck")}, "stages": 2})
            evs = [ev async for ev in core.submit_stream(
                {"model": dep["model"], "prompt": text, "max_tokens": 6})]
            await core.unload({"model": dep["model"]})
            dep2 = await core.deploy({"model": {"preset": "tiny-llama-cpu", "seed": 0}, "stages": 2})
            refused = [ev async for ev in core.submit_stream(
                {"model": dep2["model"], "prompt": text, "max_tokens": 2})]
            return evs, refused
        finally:
            for w in ws:
                await w.stop()
            await rpc.stop()

    evs, refused = asyncio.run(go())
    done = evs[-1]
    assert done["event"] == "completed", done
    assert done["tokens"] == want and done["prompt_tokens"] == len(ids)
    assert done["text"] == fast.decode(want)
    assert refused[-1]["event"] == "failed" and "no tokenizer" in refused[-1]["error"]
