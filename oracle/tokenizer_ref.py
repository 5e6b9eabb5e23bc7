"""Plain-Python restatement of the reference's tokenizer and text drivers --
test infrastructure only (the checker for ``tir_encode`` / ``tir_decode`` /
``tir_generate_text``), never part of the product path.

Follows, line for line in behaviour:
  * ``encode``  -- src/tokenizer.rs:37-120 (normalize with a leading space and
    U+2581 for every space, one symbol per char, repeatedly merge the adjacent
    pair of lowest merge rank -- the first such pair on ties -- then BOS 1, vocab
    ids, <0xXX> byte fallback, unk 0);
  * ``decode``  -- src/tokenizer.rs:122-143 (byte tokens via
    ``parse_byte_token`` :145-150, U+2581 -> space, lossy UTF-8);
  * ``generate`` / ``generate_capped`` on text -- src/lib.rs:140-314 (greedy
    ids until 13 or 2, which are not kept).
Rust's HashMap::insert keeps the last id of a repeated token and the last
rank of a repeated merge; the dicts below are filled in the same order.
"""

SPACE = "▁"


class UnknownId(Exception):
    pass


def _maps(vocab, merges):
    vmap = {}
    for i, t in enumerate(vocab):
        if isinstance(t, str):
            vmap[t] = i
    ranks = {}
    for r, m in enumerate(merges):
        if isinstance(m, str):
            ranks[m] = r
    return vmap, ranks


def encode(vocab, merges, text):
    vmap, ranks = _maps(vocab, merges)
    symbols = list((" " + text).replace(" ", SPACE))
    while True:
        best = None
        for i in range(len(symbols) - 1):
            rank = ranks.get(symbols[i] + " " + symbols[i + 1])
            if rank is not None and (best is None or rank < best[0]):
                best = (rank, i)
        if best is None:
            break
        i = best[1]
        symbols[i] = symbols[i] + symbols[i + 1]
        del symbols[i + 1]
    ids = [1]
    for s in symbols:
        if s in vmap:
            ids.append(vmap[s])
        else:
            for b in s.encode("utf-8"):
                ids.append(vmap.get(f"<0x{b:02X}>", 0))
    return ids


def _parse_byte_token(tok):
    """u8::from_str_radix(hex, 16) on "<0x" hex ">": optional '+', hex digits, <= 255."""
    if not (tok.startswith("<0x") and tok.endswith(">")) or len(tok) < 4:
        return None
    h = tok[3:-1]
    if h.startswith("+"):
        h = h[1:]
    if not h or any(c not in "0123456789abcdefABCDEF" for c in h):
        return None
    v = int(h, 16)
    return v if v <= 255 else None


def decode(vocab, ids):
    out = bytearray()
    for i in ids:
        if i < 0 or i >= len(vocab) or not isinstance(vocab[i], str):
            raise UnknownId(i)
        tok = vocab[i]
        b = _parse_byte_token(tok)
        if b is not None:
            out.append(b)
        else:
            out += tok.replace(SPACE, " ").encode("utf-8")
    return out.decode("utf-8", errors="replace")


def generate_text(orc_model, vocab, merges, text, max_new, sample):
    """src/lib.rs:140-236 on the oracle model: prompt token by token, greedy
    until 13 or 2 (at most max_new ids); returns (text, ids, margins)."""
    import numpy as np
    orc_model.reset()
    logits = None
    pos = 0
    for t in encode(vocab, merges, text):
        logits = orc_model.forward(orc_model.embed(int(t)), pos)
        pos += 1
    ids, margins = [], []
    while len(ids) < max_new:
        srt = np.sort(logits)
        margin = float(srt[-1]) - float(srt[-2])
        tok = sample(logits)
        if tok in (13, 2):
            margins.append(margin)
            break
        ids.append(tok)
        margins.append(margin)
        logits = orc_model.forward(orc_model.embed(tok), pos)
        pos += 1
    return decode(vocab, ids), ids, margins
