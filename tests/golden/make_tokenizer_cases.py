"""Regenerate tests/golden/tokenizer_cases.json from the reference's own tokenizer test cases.

The reference pins its tokenizer (h2-own-inference-engine/engine/tokenizer.js) with the token ids that Hugging Face's
tokenizer gives for the real Qwen2.5 vocabulary (h2-own-inference-engine/m1-llm/reference.json, "tokenizer" and the
chat prompts). The real vocabulary is not available to this repository's tests, so the fixture keeps each case's text
and id count: the pre-tokenizer's pieces are never merged across, so every case has at least as many ids as pieces.
Run from the repository root with the reference checkout's path (default: BASELINE.json's reference_path):

    python tests/golden/make_tokenizer_cases.py [reference checkout]
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else json.load(open(os.path.join(ROOT, "BASELINE.json")))["reference_path"]
    src = os.path.join(ref, "h2-own-inference-engine", "m1-llm", "reference.json")
    d = json.load(open(src))
    cases = [{"text": c["text"], "n_ids": len(c["ids"]), "ids": c["ids"]} for c in d["tokenizer"]]
    chats = [{"prompt": c["prompt"], "n_ids": len(c["prompt_ids"])} for c in d.get("chats", [])]
    out = {"source": "h2-own-inference-engine/m1-llm/reference.json", "model": d.get("model"), "cases": cases,
           "chat_prompts": chats}
    with open(os.path.join(HERE, "tokenizer_cases.json"), "w") as f:
        json.dump(out, f, ensure_ascii=False, indent=1)
    print(f"{len(cases)} cases, {len(chats)} chat prompts")


if __name__ == "__main__":
    main()
