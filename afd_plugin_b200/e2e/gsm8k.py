"""GSM8K accuracy against a running completions server (few-shot, exact match).

    python -m afd_plugin_b200.e2e.gsm8k --url http://127.0.0.1:8000 --data gsm8k_test.jsonl \\
        --train gsm8k_train.jsonl --shots 8 --limit 7 --threshold 0.27

The accuracy gate of the reference's end-to-end suite (first 7 samples,
8-shot, exact match >= 0.27; ``docs/design/module/e2e_testing.md:145-163``),
run against this framework's server.  Data files are GSM8K JSONL
(``{"question": ..., "answer": "... #### 42"}``) read from disk: no dataset is
downloaded.  Two scores: *strict* takes the number after ``####`` in the
completion, *flexible* the last number in it.  Needs a real checkpoint and
its tokenizer on the server to mean anything.
"""

from __future__ import annotations

import argparse
import json
import re
import sys
from concurrent.futures import ThreadPoolExecutor

import requests

_STRICT = re.compile(r"####\s*\$?\s*(-?[\d,]*\.?\d+)")
_NUMBER = re.compile(r"-?[\d,]*\.?\d+")


def load_jsonl(path: str) -> list[dict]:
    with open(path) as fh:
        return [json.loads(line) for line in fh if line.strip()]


def _norm(num: str) -> str:
    n = num.replace(",", "").rstrip(".")
    if "." in n:
        n = n.rstrip("0").rstrip(".")
    return n


def reference_answer(answer: str) -> str:
    m = _STRICT.search(answer)
    if not m:
        raise ValueError(f"GSM8K answer without '####': {answer[-80:]!r}")
    return _norm(m.group(1))


def extract_strict(text: str) -> str | None:
    m = _STRICT.search(text)
    return _norm(m.group(1)) if m else None


def extract_flexible(text: str) -> str | None:
    nums = _NUMBER.findall(text)
    return _norm(nums[-1]) if nums else None


def build_prompt(shots: list[dict], question: str) -> str:
    """``Question: ...\\nAnswer: ...`` blocks, then the open question."""
    parts = [f"Question: {s['question']}\nAnswer: {s['answer']}\n\n" for s in shots]
    return "".join(parts) + f"Question: {question}\nAnswer:"


def _truncate(text: str) -> str:
    """The model's answer ends where it starts the next few-shot block."""
    for stop in ("\n\nQuestion:", "Question:"):
        i = text.find(stop)
        if i >= 0:
            text = text[:i]
    return text


def evaluate(url: str, data: list[dict], shots: list[dict], *, limit: int | None = None, max_tokens: int = 256,
             concurrency: int = 8, timeout_s: float = 600.0) -> dict:
    items = data[:limit] if limit else data
    endpoint = url.rstrip("/") + "/v1/completions"

    def one(item):
        r = requests.post(endpoint, json={"prompt": build_prompt(shots, item["question"]), "max_tokens": max_tokens,
                                          "stop": ["Question:"]}, timeout=timeout_s)
        r.raise_for_status()
        return _truncate(r.json()["choices"][0]["text"])

    with ThreadPoolExecutor(max(1, concurrency)) as ex:
        outs = list(ex.map(one, items))
    gold = [reference_answer(it["answer"]) for it in items]
    strict = sum(extract_strict(o) == g for o, g in zip(outs, gold))
    flexible = sum(extract_flexible(o) == g for o, g in zip(outs, gold))
    n = max(1, len(items))
    return {"n": len(items), "exact_match_strict": strict / n, "exact_match_flexible": flexible / n,
            "shots": len(shots)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--url", default="http://127.0.0.1:8000")
    ap.add_argument("--data", required=True, help="GSM8K test split as JSONL")
    ap.add_argument("--train", default=None, help="few-shot examples as JSONL (default: the head of --data)")
    ap.add_argument("--shots", type=int, default=8)
    ap.add_argument("--limit", type=int, default=7)
    ap.add_argument("--max-tokens", type=int, default=256)
    ap.add_argument("--threshold", type=float, default=0.27, help="gate on the flexible exact match")
    ap.add_argument("--output", default=None)
    args = ap.parse_args(argv)
    data = load_jsonl(args.data)
    pool = load_jsonl(args.train) if args.train else data
    shots = pool[: args.shots]
    if not args.train:
        data = data[args.shots:]
    res = evaluate(args.url, data, shots, limit=args.limit, max_tokens=args.max_tokens)
    res["threshold"] = args.threshold
    res["gate"] = "pass" if res["exact_match_flexible"] >= args.threshold else "fail"
    print(json.dumps(res), flush=True)
    if args.output:
        with open(args.output, "w") as fh:
            json.dump(res, fh)
    return 0 if res["gate"] == "pass" else 1


if __name__ == "__main__":
    sys.exit(main())
