"""Byte-level BPE tokenizer built from a GGUF's vocabulary and merge table:
hs-engine tok.rs (Tokenizer::from_gguf / encode / decode_bytes /
pretokenize), host-side like the reference's.

The Qwen2 pre-tokenizer pattern

    (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}
      | ?[^\\s\\p{L}\\p{N}]+[\\r\\n]*|\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+

is a scanner that tries the alternatives in order at each position, with the
reference's character classes: a letter is Rust's char::is_alphabetic (the
Unicode Alphabetic property), a number char::is_numeric (general categories
Nd, Nl, No), whitespace char::is_whitespace (White_Space). Those properties
come from the `regex` module's Unicode tables (\\p{Alphabetic}, \\p{N},
\\p{White_Space}), whose Unicode version can differ from the Rust standard
library's in characters assigned after it.
"""
import struct
from functools import lru_cache

import regex

_ALPHA = regex.compile(r"\p{Alphabetic}")
_NUM = regex.compile(r"\p{N}")
_WS = regex.compile(r"\p{White_Space}")


@lru_cache(maxsize=65536)
def is_letter(c):
    return _ALPHA.match(c) is not None


@lru_cache(maxsize=65536)
def is_number(c):
    return _NUM.match(c) is not None


@lru_cache(maxsize=65536)
def is_space(c):
    return _WS.match(c) is not None


def is_nl(c):
    return c == "\r" or c == "\n"


def byte_to_unicode():
    """GPT-2's byte -> printable character table and its inverse (tok.rs:28-52)."""
    direct = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    b2u = [""] * 256
    used = [False] * 256
    for b in direct:
        b2u[b] = chr(b)
        used[b] = True
    n = 0
    for b in range(256):
        if not used[b]:
            b2u[b] = chr(256 + n)
            n += 1
    return b2u, {u: b for b, u in enumerate(b2u)}


def pretokenize(text):
    """The pieces of `text` under the Qwen2 pattern (tok.rs:212-345)."""
    c = text
    n = len(c)
    out = []
    i = 0
    while i < n:
        start = i
        # 1. contractions, case-insensitive
        if c[i] == "'" and i + 1 < n:
            two = c[i + 1:min(i + 3, n)].lower()
            if two.startswith(("re", "ve", "ll")):
                ln = 3
            elif two[:1] in ("s", "t", "m", "d"):
                ln = 2
            else:
                ln = 0
            if ln:
                out.append(c[i:i + ln])
                i += ln
                continue
        # 2. [^\r\n\p{L}\p{N}]?\p{L}+ (the optional char taken greedily,
        #    given back when no letter follows)
        j = i
        if not is_nl(c[j]) and not is_letter(c[j]) and not is_number(c[j]):
            j += 1
        if j < n and is_letter(c[j]):
            while j < n and is_letter(c[j]):
                j += 1
            out.append(c[i:j])
            i = j
            continue
        if is_letter(c[i]):
            j = i
            while j < n and is_letter(c[j]):
                j += 1
            out.append(c[i:j])
            i = j
            continue
        # 3. \p{N}, one at a time
        if is_number(c[i]):
            out.append(c[i])
            i += 1
            continue
        # 4.  ?[^\s\p{L}\p{N}]+[\r\n]*
        j = i
        if c[j] == " ":
            j += 1
        sym = j
        while j < n and not is_space(c[j]) and not is_letter(c[j]) and not is_number(c[j]):
            j += 1
        if j > sym:
            while j < n and is_nl(c[j]):
                j += 1
            out.append(c[i:j])
            i = j
            continue
        if is_space(c[i]):
            run = i
            while run < n and is_space(c[run]):
                run += 1
            # 5. \s*[\r\n]+: the longest \s* prefix that still leaves a newline
            k = run
            while True:
                if k < n and is_nl(c[k]):
                    e = k
                    while e < n and is_nl(c[e]):
                        e += 1
                    out.append(c[i:e])
                    i = e
                    break
                if k == i:
                    break
                k -= 1
            if i != start:
                continue
            # 6. \s+(?!\S): the run keeps its last char only at the end
            if run == n:
                out.append(c[i:run])
                i = run
                continue
            if run - i > 1:
                out.append(c[i:run - 1])
                i = run - 1
                continue
            # 7. \s+
            out.append(c[i:run])
            i = run
            continue
        # a lone character nothing matched
        out.append(c[i])
        i += 1
    return out


def _gguf_metadata(path):
    """The metadata key/value pairs of a GGUF file (gguf.rs:225-296): strings,
    string and i32 arrays as lists, numbers as ints/floats."""
    with open(path, "rb") as f:
        data = f.read(1 << 20)

        def take(p, k):
            nonlocal data
            while p + k > len(data):
                more = f.read(max(1 << 20, p + k - len(data)))
                if not more:
                    raise ValueError("truncated GGUF metadata")
                data += more
            return data[p:p + k], p + k

        b, p = take(0, 24)
        magic, version, n_tensors, n_kv = struct.unpack("<IIQQ", b)
        if magic != 0x46554747:
            raise ValueError("not a GGUF file")
        scal = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}

        def string(p):
            b, p = take(p, 8)
            ln = struct.unpack("<Q", b)[0]
            b, p = take(p, ln)
            return b.decode("utf-8", errors="replace"), p

        def value(p, ty):
            if ty == 8:
                return string(p)
            if ty == 9:
                b, p = take(p, 12)
                ety, ln = struct.unpack("<IQ", b)
                vals = []
                for _ in range(ln):
                    v, p = value(p, ety)
                    vals.append(v)
                return vals, p
            fmt = scal.get(ty)
            if fmt is None:
                raise ValueError(f"bad GGUF value type {ty}")
            b, p = take(p, struct.calcsize(fmt))
            return struct.unpack(fmt, b)[0], p

        meta = {}
        for _ in range(n_kv):
            key, p = string(p)
            b, p = take(p, 4)
            v, p = value(p, struct.unpack("<I", b)[0])
            meta[key] = v
        return meta


class Tokenizer:
    """Tokenizer over an explicit vocabulary and merge table, or from a GGUF
    (Tokenizer::from_gguf, tok.rs:55-97)."""

    def __init__(self, vocab, merges, token_types=None, eos=0, bos=None):
        self.vocab = list(vocab)
        self.ids = {}
        for i, t in enumerate(self.vocab):
            self.ids.setdefault(t, i)
        self.ranks = {}
        for r, m in enumerate(merges):
            sp = m.find(" ")
            if sp >= 0:
                self.ranks[(m[:sp], m[sp + 1:])] = r  # a repeated pair keeps its last rank (HashMap::insert)
        types = list(token_types or [])
        self.specials = [(t, i) for i, t in enumerate(self.vocab)
                         if (types[i] if i < len(types) else 1) == 3 and t.startswith("<|")]
        self.specials.sort(key=lambda x: -len(x[0]))  # longest match first (a stable sort, like Rust's)
        self.b2u, self.u2b = byte_to_unicode()
        self.eos = eos
        self.bos = bos

    @classmethod
    def from_gguf(cls, path):
        meta = _gguf_metadata(path)
        vocab = meta["tokenizer.ggml.tokens"]
        merges = meta["tokenizer.ggml.merges"]
        types = meta.get("tokenizer.ggml.token_type") or []
        eos = int(meta["tokenizer.ggml.eos_token_id"])
        bos = None
        if "tokenizer.ggml.bos_token_id" in meta and meta.get("tokenizer.ggml.add_bos_token") is True:
            bos = int(meta["tokenizer.ggml.bos_token_id"])
        return cls(vocab, merges, types, eos, bos)

    def vocab_size(self):
        return len(self.vocab)

    def id_of(self, s):
        return self.ids.get(s)

    def encode(self, text):
        """Token ids of `text`, control tokens like <|im_start|> matched
        literally (tok.rs:99-135)."""
        out = [] if self.bos is None else [self.bos]
        rest = text
        while rest:
            hit = None
            for s, i in self.specials:
                at = rest.find(s)
                if at >= 0 and (hit is None or at < hit[0]):
                    hit = (at, s, i)
            if hit is None:
                self._encode_ordinary(rest, out)
                break
            at, s, i = hit
            if at > 0:
                self._encode_ordinary(rest[:at], out)
            out.append(i)
            rest = rest[at + len(s):]
        return out

    def _encode_ordinary(self, text, out):
        for piece in pretokenize(text):
            sym = [self.b2u[b] for b in piece.encode("utf-8")]
            self._bpe(sym)
            for s in sym:
                i = self.ids.get(s)
                if i is None:
                    raise ValueError(f"token {s!r} is not in the vocabulary")
                out.append(i)

    def _bpe(self, sym):
        """Merge the lowest-ranked adjacent pair until none is in the table
        (tok.rs:152-167; the first of equal ranks wins)."""
        while True:
            best = None
            for i in range(len(sym) - 1):
                r = self.ranks.get((sym[i], sym[i + 1]))
                if r is not None and (best is None or r < best[0]):
                    best = (r, i)
            if best is None:
                return
            i = best[1]
            sym[i:i + 2] = [sym[i] + sym[i + 1]]

    def decode_bytes(self, ids):
        """Bytes of the ids; a character with no byte encoding (a control
        token's) is emitted as its UTF-8 (tok.rs:169-186)."""
        out = bytearray()
        for i in ids:
            if i >= len(self.vocab):
                continue
            for ch in self.vocab[i]:
                b = self.u2b.get(ch)
                if b is None:
                    out += ch.encode("utf-8")
                else:
                    out.append(b)
        return bytes(out)

    def decode(self, ids):
        return self.decode_bytes(ids).decode("utf-8", errors="replace")

    def token_text(self, i):
        return self.decode([i])
