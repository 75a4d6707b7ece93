"""Text in, text out through the CUDA engine: LLM.chat (llm.js:56-82) with the host tokenizer (tokenizer.py) on a
seeded model whose GGUF carries a byte-level BPE vocabulary trained here (bpe_vocab.py).

The reply's token ids are the engine's greedy continuation of the ChatML prompt (the same ids as generate_ids), the
streamed text is their decoding, and a second turn reuses the cached prefix (llm.js:45-54)."""
import pytest
import torch

from e2e_browser_voice_agent_b200 import synth
from e2e_browser_voice_agent_b200.llm import LLM
from e2e_browser_voice_agent_b200.tokenizer import chat_prompt

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model_path(tmp_path_factory):
    pytest.importorskip("tokenizers")
    import bpe_vocab
    _, tok = bpe_vocab.train()
    cfg = dict(synth.CONFIGS["small"], vocab=len(tok[0]))
    path = str(tmp_path_factory.mktemp("bpe") / "small-bpe.gguf")
    synth.build(path, cfg, seed=3, tokenizer=tok)
    return path


def test_chat_streams_the_greedy_reply_and_reuses_the_cache(model_path):
    assert torch.cuda.is_available()
    llm = LLM.load(model_path, ctx=192, prefill_chunk=16)
    assert llm.tok is not None
    msgs = [{"role": "user", "content": "hello there, how are you?"}]
    text = "".join(llm.chat(msgs, max_tokens=12))
    st = llm.stats
    ids = st["ids"]
    assert 0 < len(ids) <= 12 and st["reused"] == 0 and st["prefilled"] == st["prompt_tokens"]
    assert llm.tok.decode(ids).startswith(text)  # (a character split at the end is held back by the stream)
    ref = LLM.load(model_path, ctx=192, prefill_chunk=16)
    prompt_ids = ref.tok.encode(chat_prompt(msgs))
    assert prompt_ids == llm.tok.encode(chat_prompt(msgs))
    assert ref.generate_ids(prompt_ids, len(ids)) == ids
    # the next turn: the history (prompt + reply) stays in the cache, only the new message runs
    msgs2 = msgs + [{"role": "assistant", "content": text}, {"role": "user", "content": "and then?"}]
    list(llm.chat(msgs2, max_tokens=4))
    assert llm.stats["reused"] > 0 and llm.stats["prefilled"] < llm.stats["prompt_tokens"]
    llm.be.destroy()
    ref.be.destroy()
