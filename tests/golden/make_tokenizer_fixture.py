#!/usr/bin/env python3
"""Generate the tokenizer fixture under tests/golden/tok/ (run from the repo root).

GPT-2's vocab.json and merges.txt are not available offline, so this trains a
small byte-level BPE vocabulary (bytes_to_unicode symbols + 400 merges) on a
seeded synthetic corpus and writes it in GPT-2's file formats (JSON with
\\u escapes, "#version" merges header).  The expected ids and decoded bytes of
each case text come from the REFERENCE's own tokenizer.c (compiled into
oracle/_ref/libref_main.so by oracle/Makefile); the script refuses to run
without it.

    python tests/golden/make_tokenizer_fixture.py
"""
import collections
import json
import os
import random
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
OUT = os.path.join(HERE, "tok")


def bytes_to_unicode():
    keep = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    cps, extra = {}, 0
    for b in range(256):
        if b in keep:
            cps[b] = b
        else:
            cps[b] = 256 + extra
            extra += 1
    return {b: chr(c) for b, c in cps.items()}


B2U = bytes_to_unicode()


def corpus(rng):
    syll = ["ka", "to", "ri", "mu", "ne", "sa", "lo", "vi", "pe", "du", "an", "er", "th", "in", "on", "st", "qu", "ou"]
    words = ["".join(rng.choice(syll) for _ in range(rng.randint(1, 4))) for _ in range(300)]
    weights = [1.0 / (i + 1) for i in range(len(words))]
    extras = ["'s", "'re", "'ve", "'ll", "'t", "'d", "'m", "123", "2024", "3.14", "!!", "?", ",", ".", "--", "()",
              "café", "über", "日本", "naïve", "\U0001F642"]
    parts = []
    for _ in range(6000):
        w = rng.choices(words, weights)[0] if rng.random() < 0.85 else rng.choice(extras)
        if rng.random() < 0.1:
            w = w.capitalize()
        parts.append(w)
        parts.append(rng.choice([" ", " ", " ", " ", "\n", "  ", ", ", ". "]))
    return "".join(parts)


def pretokens(text):
    """Coarse word split for training only (any split yields valid merges)."""
    out, cur = [], ""
    for ch in text:
        if ch == " " and cur and not cur.isspace():
            out.append(cur)
            cur = ch
        else:
            cur += ch
    if cur:
        out.append(cur)
    return out


def train(text, n_merges):
    counts = collections.Counter(pretokens(text))
    seqs = {w: [B2U[b] for b in w.encode()] for w in counts}
    merges = []
    for _ in range(n_merges):
        pairs = collections.Counter()
        for w, c in counts.items():
            s = seqs[w]
            for a, b in zip(s, s[1:]):
                pairs[(a, b)] += c
        if not pairs:
            break
        best = max(pairs.items(), key=lambda kv: (kv[1], kv[0]))[0]
        merges.append(best)
        for w in counts:
            s, out, i = seqs[w], [], 0
            while i < len(s):
                if i + 1 < len(s) and (s[i], s[i + 1]) == best:
                    out.append(s[i] + s[i + 1])
                    i += 2
                else:
                    out.append(s[i])
                    i += 1
            seqs[w] = out
    return merges


CASES = [
    "Hello world", "hello  world", " leading space", "trailing space ", "tabs\tand\nnewlines\r\n",
    "I'm sure they're here, we've seen it; you'll see what's up.", "'twas", "don't", "o'clock", "' s",
    "numbers 123 4567 89.0 and 2024-01-01", "punct!!! ??? ... ,,, ;;; ()[]{}", " !x", "aéb café naïve",
    "日本語の文", "emoji \U0001F642\U0001F680 end", "", " ", "   ", "\n\n\n", "x" * 600, "z" * 40,
    "MiXeD CaSe WoRdS", "kato rimu nesa lovi pedu", "anerthinonstqu outh'll", "tab\t\ttab", " nbsp ",
]


def main():
    import oracle
    if not oracle.ref_available():
        sys.exit("oracle/_ref/libref_main.so is missing: run make -C oracle with the reference sources present")
    rng = random.Random(20241201)
    text = corpus(rng)
    merges = train(text, 400)
    symbols = [B2U[b] for b in range(256)]
    vocab = {s: i for i, s in enumerate(symbols)}
    for a, b in merges:
        if a + b not in vocab:
            vocab[a + b] = len(vocab)
    vocab["<|endoftext|>"] = len(vocab)
    vocab["\U0001F642"] = len(vocab)   # a surrogate-pair escape in the JSON; decodes to '?'
    os.makedirs(OUT, exist_ok=True)
    with open(os.path.join(OUT, "vocab.json"), "w") as f:
        json.dump(vocab, f, ensure_ascii=True)
    with open(os.path.join(OUT, "merges.txt"), "w", encoding="utf-8") as f:
        f.write("#version: 0.2\n")
        for a, b in merges:
            f.write(f"{a} {b}\n")
    ref = oracle.RefTokenizer(OUT)
    cases = []
    for i, t in enumerate(CASES + [text[k * 400:(k + 1) * 400] for k in range(12)]):
        data = t.encode()
        ids = ref.encode(data)
        cases.append({"text_hex": data.hex(), "ids": ids, "decoded_hex": ref.decode(ids).hex(),
                      "ids_max8": ref.encode(data, 8)})
    ref.close()
    with open(os.path.join(OUT, "cases.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_tokenizer_fixture.py", "n_merges": len(merges),
                   "vocab_size": len(vocab), "cases": cases}, f, indent=0)
    print(f"wrote {len(vocab)} tokens, {len(merges)} merges, {len(cases)} cases to {OUT}")


if __name__ == "__main__":
    main()
