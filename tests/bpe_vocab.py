"""A byte-level BPE vocabulary trained here (Hugging Face `tokenizers`, Qwen2's pre-tokenizer) on a synthetic corpus,
for the tokenizer tests and the text-in / text-out engine test (the real Qwen2.5 vocabulary is not available)."""
import json
import random

from e2e_browser_voice_agent_b200 import tokenizer as T

SPECIAL = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]


def corpus(rng, n):
    alphabet = ("abcdefghijklmnopqrstuvwxyz" * 3 + "ABCDEFGHIJ" + "0123456789" + " " * 20 + ".,;:!?'\"()-\n\t" +
                "éüñçåøæ" + "日本語中文🙂👍")
    words = ["".join(rng.choice(alphabet[:26]) for _ in range(rng.randint(1, 7))) for _ in range(300)]
    out = []
    for _ in range(n):
        s = []
        for _ in range(rng.randint(1, 12)):
            r = rng.random()
            s.append(rng.choice(words) if r < 0.6 else "".join(rng.choice(alphabet) for _ in range(rng.randint(1, 4))))
            s.append(rng.choice([" ", " ", " ", "  ", "\n", "", "'s ", "\r\n", "\t"]))
        out.append("".join(s))
    return out


def train(vocab_size=700, seed=7):
    """(hf tokenizer, (tokens, merges, token types)) of a byte-level BPE trained on the synthetic corpus."""
    import tokenizers
    from tokenizers import Regex, Tokenizer, decoders, models, pre_tokenizers, trainers
    hf = Tokenizer(models.BPE())
    hf.normalizer = tokenizers.normalizers.NFC()
    hf.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(T.PRE.pattern), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    hf.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=vocab_size, special_tokens=SPECIAL, show_progress=False,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    hf.train_from_iterator(corpus(random.Random(seed), 3000), trainer)
    spec = json.loads(hf.to_str())
    vocab = spec["model"]["vocab"]
    tokens = [None] * len(vocab)
    for s, i in vocab.items():
        tokens[i] = s
    merges = [m if isinstance(m, str) else " ".join(m) for m in spec["model"]["merges"]]
    types = [3 if t in SPECIAL else 1 for t in tokens]
    return hf, (tokens, merges, types)
