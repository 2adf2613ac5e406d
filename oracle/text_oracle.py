"""Text front end of the reference, restated in Python — TEST INFRASTRUCTURE.

Only tests/ may use this module; it is the CPU checker for the C++ front end
(needle-rs_b200/csrc/frontend.cpp), never a product path.  Each function
restates the reference step for step, with the file:line it follows:

  Vocab.parse / encode / encode_bpe / encode_greedy / decode_ids
      crates/needle-infer/src/tokenizer.rs:42-216 (BPE as the reference writes
      it: rescan every adjacent pair after each merge, first maximum wins)
  normalize_sp                    tokenizer.rs:218-236
  to_snake_case                   tokenizer.rs:248-292 (ASCII and no-case
                                  non-ASCII characters, as the C++ front end)
  parse_tools_json and helpers    crates/needle-infer/src/constrained.rs:378-689
  normalize_tools_json / compact_json / restore_tool_names
                                  crates/needle-infer/src/engine.rs:354-546
  Trie / JsonStateMachine / ConstrainedDecoder
                                  constrained.rs:15-375
  encoder_input                   engine.rs:231-266 (run_impl's truncation)
Strings are handled as Python str for text and bytes for the state machine.
"""
import math

SP = "▁"
PAD, EOS, BOS, UNK, TOOL_CALL, TOOLS = 0, 1, 2, 3, 4, 5
_WS = set([0x09, 0x0A, 0x0B, 0x0C, 0x0D, 0x20, 0x85, 0xA0, 0x1680, 0x2028, 0x2029, 0x202F, 0x205F, 0x3000] +
          list(range(0x2000, 0x200B)))


def is_ws(ch):
    return ord(ch) in _WS


def rtrim(s):
    i = len(s)
    while i > 0 and is_ws(s[i - 1]):
        i -= 1
    return s[:i]


def ltrim(s):
    i = 0
    while i < len(s) and is_ws(s[i]):
        i += 1
    return s[i:]


def trim(s):
    return rtrim(ltrim(s))


def _parse_f32(t):
    body = t[1:] if t[:1] in "+-" else t
    low = body.lower()
    if low in ("inf", "infinity"):
        return -math.inf if t[:1] == "-" else math.inf
    if low == "nan":
        return math.nan
    if not body or not any(c.isdigit() for c in body) or any(c not in "0123456789.eE+-" for c in body):
        return 0.0
    try:
        import numpy as np
        return float(np.float32(float(t)))
    except ValueError:
        return 0.0


def _lines(content):
    # str::lines: split on '\n', drop one '\r' before it, no empty last line
    out = []
    i = 0
    while i < len(content):
        j = content.find("\n", i)
        if j < 0:
            out.append(content[i:])
            break
        line = content[i:j]
        if line.endswith("\r"):
            line = line[:-1]
        out.append(line)
        i = j + 1
    return out


class Vocab:
    def __init__(self, content):
        self.id_to_piece, self.piece_to_id, self.scores = [], {}, []
        has_scores = False
        self.max_piece_bytes = 0
        for line in _lines(content):
            pid = len(self.id_to_piece)
            tab = line.find("\t")
            if tab >= 0:
                has_scores = True
                piece, score = line[:tab], _parse_f32(trim(line[tab + 1:]))
            else:
                piece, score = line, 0.0
            self.max_piece_bytes = max(self.max_piece_bytes, len(piece.encode()))
            self.piece_to_id[piece] = pid
            self.id_to_piece.append(piece)
            self.scores.append(score)
        if not has_scores:
            self.scores = []

    def encode(self, text):
        text = trim(text)
        if not text:
            return []
        norm = normalize_sp(text)
        return self.encode_greedy(norm.encode()) if not self.scores else self.encode_bpe(norm)

    def encode_bpe(self, norm):
        pieces, strings = [], []
        for c in norm:
            if c in self.piece_to_id:
                strings.append(c)
                pieces.append(self.piece_to_id[c])
            else:
                for b in c.encode():
                    fb = "<0x%02X>" % b
                    strings.append(fb)
                    pieces.append(self.piece_to_id.get(fb, UNK))
        while True:
            best_score, best_i, best_id = -math.inf, None, 0
            for i in range(len(strings) - 1):
                merged = strings[i] + strings[i + 1]
                pid = self.piece_to_id.get(merged)
                if pid is not None:
                    score = self.scores[pid]
                    if score > best_score:
                        best_score, best_i, best_id = score, i, pid
            if best_i is None:
                break
            strings[best_i] = strings[best_i] + strings[best_i + 1]
            del strings[best_i + 1]
            pieces[best_i] = best_id
            del pieces[best_i + 1]
        return pieces

    def encode_greedy(self, b):
        n, ids, pos = len(b), [], 0
        cont = lambda k: (b[k] & 0xC0) == 0x80  # noqa: E731
        while pos < n:
            end = min(pos + self.max_piece_bytes, n)
            while end > pos and end < n and cont(end):
                end -= 1
            found = False
            while end > pos:
                try:
                    piece = b[pos:end].decode()
                    pid = self.piece_to_id.get(piece)
                except UnicodeDecodeError:
                    pid = None
                if pid is not None:
                    ids.append(pid)
                    pos = end
                    found = True
                    break
                end -= 1
                while end > pos and cont(end):
                    end -= 1
            if not found:
                ids.append(self.piece_to_id.get("<0x%02X>" % b[pos], UNK))
                pos += 1
        return ids

    def decode_ids(self, ids):
        out = "".join(self.id_to_piece[i].replace(SP, " ") for i in ids if i < len(self.id_to_piece))
        return ltrim(out)

    def piece_text(self, i):
        return self.id_to_piece[i].replace(SP, " ") if i < len(self.id_to_piece) else ""


def normalize_sp(text):
    out, prev = [SP], False
    for c in text:
        if is_ws(c):
            if not prev:
                out.append(SP)
                prev = True
        else:
            out.append(c)
            prev = False
    return "".join(out)


def to_snake_case(name):
    up = lambda c: "A" <= c <= "Z"  # noqa: E731
    lo = lambda c: "a" <= c <= "z"  # noqa: E731
    dg = lambda c: "0" <= c <= "9"  # noqa: E731
    an = lambda c: up(c) or lo(c) or dg(c) or ord(c) >= 0x80  # noqa: E731
    out, prev_us, prev_up = [], False, False
    ch = list(name)
    n = len(ch)
    for i, c in enumerate(ch):
        if an(c) or c == "_":
            if c == "_":
                if not prev_us and out:
                    out.append("_")
                    prev_us = True
                prev_up = False
            elif up(c):
                prev_lower = i > 0 and (lo(ch[i - 1]) or dg(ch[i - 1]))
                next_lower = i + 1 < n and lo(ch[i + 1])
                if i > 0 and not prev_us and (prev_lower or (prev_up and next_lower)):
                    out.append("_")
                out.append(c.lower())
                prev_us, prev_up = False, True
            else:
                out.append(c)
                prev_us, prev_up = False, False
        else:
            if not prev_us and out:
                out.append("_")
                prev_us = True
            prev_up = False
    s = "".join(out)
    while s.endswith("_"):
        s = s[:-1]
    return s


# ── tool JSON (byte level, constrained.rs:378-689) ──────────────────────────

_AWS = b" \t\n\x0c\r"


def _find_matching(b, start, op, cl):
    depth, in_str, esc = 0, False, False
    for i in range(start, len(b)):
        c = b[i]
        if in_str:
            if esc:
                esc = False
            elif c == 0x5C:
                esc = True
            elif c == 0x22:
                in_str = False
        elif c == 0x22:
            in_str = True
        elif c == op:
            depth += 1
        elif c == cl:
            depth = max(depth - 1, 0)
            if depth == 0:
                return i
    return max(len(b) - 1, 0)


def _extract_string(obj, field):
    key = b'"' + field + b'":"'
    pos = obj.find(key)
    if pos < 0:
        return None
    s = pos + len(key)
    esc = False
    for i in range(s, len(obj)):
        if esc:
            esc = False
        elif obj[i] == 0x5C:
            esc = True
        elif obj[i] == 0x22:
            return obj[s:i]
    return None


def _extract_object(obj, field):
    key = b'"' + field + b'":'
    pos = obj.find(key)
    if pos < 0:
        return None
    after = ltrim(obj[pos + len(key):].decode()).encode()
    if not after or after[0] != 0x7B:
        return None
    end = _find_matching(after, 0, 0x7B, 0x7D)
    return after[:end + 1]


def _skip_value(b, i):
    if i >= len(b):
        return i
    if b[i] == 0x7B:
        return _find_matching(b, i, 0x7B, 0x7D) + 1
    if b[i] == 0x5B:
        return _find_matching(b, i, 0x5B, 0x5D) + 1
    if b[i] == 0x22:
        i += 1
        esc = False
        while i < len(b):
            if esc:
                esc = False
            elif b[i] == 0x5C:
                esc = True
            elif b[i] == 0x22:
                return i + 1
            i += 1
        return i
    while i < len(b) and b[i] not in b",}]":
        i += 1
    return i


def _keys(b, object_values_only):
    keys, i = [], 0
    if i < len(b) and b[i] == 0x7B:
        i += 1
    while i < len(b):
        while i < len(b) and (b[i] == 0x2C or b[i] in _AWS):
            i += 1
        if i >= len(b) or b[i] == 0x7D:
            break
        if b[i] != 0x22:
            i += 1
            continue
        i += 1
        ks, esc = i, False
        while i < len(b):
            if esc:
                esc = False
            elif b[i] == 0x5C:
                esc = True
            elif b[i] == 0x22:
                break
            i += 1
        key = b[ks:i]
        i += 1
        while i < len(b) and b[i] != 0x3A:
            i += 1
        i += 1
        while i < len(b) and b[i] in _AWS:
            i += 1
        if object_values_only:
            if i < len(b) and b[i] == 0x7B:
                if key:
                    keys.append(key)
                i = _find_matching(b, i, 0x7B, 0x7D) + 1
            else:
                i = _skip_value(b, i)
        else:
            if key:
                keys.append(key)
            i = _skip_value(b, i)
    return keys


def parse_tools_json(json_text):
    """-> list of (name, snake_name, param_keys) with str values."""
    b = json_text.encode()
    tools, i, n = [], 0, len(b)
    while i < n and b[i] not in b"[{":
        i += 1
    if i >= n:
        return tools
    if b[i] == 0x5B:
        i += 1
    while i < n:
        while i < n and (b[i] == 0x2C or b[i] in _AWS):
            i += 1
        if i >= n or b[i] == 0x5D:
            break
        if b[i] != 0x7B:
            i += 1
            continue
        end = _find_matching(b, i, 0x7B, 0x7D)
        obj = b[i:end + 1]
        name = _extract_string(obj, b"name")
        if name is not None:
            params = _extract_object(obj, b"parameters")
            keys = []
            if params is not None:
                props = _extract_object(params, b"properties")
                keys = _keys(props, False) if props is not None else _keys(params, True)
            nm = name.decode()
            tools.append((nm, to_snake_case(nm), [k.decode() for k in keys]))
        i = end + 1
    return tools


def _rename(json_text, pairs):
    if not pairs:
        return json_text
    b = json_text.encode()
    out, i, flushed, n = bytearray(), 0, 0, len(b)
    while i < n:
        if b[i:i + 6] == b'"name"':
            out += b[flushed:i] + b'"name"'
            i += 6
            while i < n and b[i] in _AWS:
                i += 1
            if i < n and b[i] == 0x3A:
                out += b":"
                i += 1
            while i < n and b[i] in _AWS:
                i += 1
            if i < n and b[i] == 0x22:
                out += b'"'
                i += 1
                vs = i
                while i < n:
                    if b[i] == 0x5C:
                        i += 2
                        continue
                    if b[i] == 0x22:
                        break
                    i += 1
                i = min(i, n)
                val = b[vs:i]
                rep = val
                for a, c in pairs:
                    if a == val:
                        rep = c
                        break
                out += rep
                if i < n:
                    out += b'"'
                    i += 1
            flushed = i
        else:
            i += 1
    out += b[flushed:]
    return out.decode()


def normalize_tools_json(json_text, tools):
    return _rename(json_text, [(t[0].encode(), t[1].encode()) for t in tools if t[0] != t[1]])


def restore_tool_names(text, tools):
    pairs = [(t[1].encode(), t[0].encode()) for t in tools if t[0] != t[1]]
    pairs.sort(key=lambda p: -len(p[0]))  # stable, longest snake name first
    return _rename(text, pairs)


def compact_json(s):
    out, in_str, it = [], False, iter(s)
    for ch in it:
        if in_str:
            out.append(ch)
            if ch == "\\":
                nxt = next(it, None)
                if nxt is not None:
                    out.append(nxt)
            elif ch == '"':
                in_str = False
        elif ch == '"':
            in_str = True
            out.append('"')
        elif ch in " \t\n\x0c\r":
            pass
        else:
            out.append(ch)
    return "".join(out)


# ── constrained decoding (constrained.rs:15-375) ────────────────────────────

class Trie:
    def __init__(self):
        self.children, self.terminal = [{}], [False]

    def insert(self, s):
        cur = 0
        for b in s:
            nxt = self.children[cur].get(b)
            if nxt is None:
                nxt = len(self.children)
                self.children.append({})
                self.terminal.append(False)
                self.children[cur][b] = nxt
            cur = nxt
        self.terminal[cur] = True

    def advance(self, node, s):
        cur = node
        for b in s:
            cur = self.children[cur].get(b)
            if cur is None:
                return None
        return cur

    def token_valid(self, bts, node):
        cur = node
        for b in bts:
            if b == 0x22:
                return self.terminal[cur]
            cur = self.children[cur].get(b)
            if cur is None:
                return False
        return True


FREE, IN_NAME, IN_ARG_KEY = 0, 1, 2


class JsonStateMachine:
    def __init__(self):
        self.state, self.current_function, self.buf = FREE, b"", b""
        self.in_arguments, self.arguments_depth, self.nesting = False, 0, 0
        self.in_string, self.prev_escape, self.tail = False, False, b""

    def feed_byte(self, b):
        if self.state in (IN_NAME, IN_ARG_KEY):
            if b == 0x22:
                if self.state == IN_NAME:
                    self.current_function = self.buf
                self.buf = b""
                self.state = FREE
            else:
                self.buf += bytes([b])
            return
        self.tail = (self.tail + bytes([b]))[-13:]
        if self.in_string:
            if self.prev_escape:
                self.prev_escape = False
                return
            if b == 0x5C:
                self.prev_escape = True
                return
            if b == 0x22:
                self.in_string = False
            return
        if b in (0x7B, 0x5B):
            self.nesting += 1
        elif b in (0x7D, 0x5D):
            self.nesting = max(self.nesting - 1, 0)
            if b == 0x7D and self.in_arguments and self.nesting < self.arguments_depth:
                self.in_arguments = False
            return
        if not self.in_arguments and self.tail.endswith(b'"name":"'):
            self.state, self.buf = IN_NAME, b""
            return
        if self.tail.endswith(b'"arguments":{'):
            self.in_arguments, self.arguments_depth = True, self.nesting
            return
        t = self.tail
        if (self.in_arguments and self.nesting == self.arguments_depth and len(t) >= 2 and t[-2] in b"{,"
                and t[-1] == 0x22):
            self.state, self.buf = IN_ARG_KEY, b""
            return
        if b == 0x22 and len(t) >= 2 and t[-2] == 0x3A:
            self.in_string = True

    def feed(self, bts):
        for b in bts:
            self.feed_byte(b)


class ConstrainedDecoder:
    def __init__(self, tools, vocab):
        self.name_trie, self.param_tries = Trie(), {}
        for _, snake, keys in tools:
            self.name_trie.insert(snake.encode())
            t = Trie()
            for k in keys:
                t.insert(k.encode())
            self.param_tries[snake.encode()] = t
        self.texts = [vocab.piece_text(i).encode() for i in range(len(vocab.id_to_piece))]
        self.sm = JsonStateMachine()

    def update(self, tok):
        if tok < len(self.texts):
            self.sm.feed(self.texts[tok])

    def allowed(self, vocab_size):
        """None when unconstrained, else the list of allowed token ids."""
        sm = self.sm
        if sm.state == IN_NAME:
            trie = self.name_trie
        elif sm.state == IN_ARG_KEY:
            trie = self.param_tries.get(sm.current_function)
            if trie is None:
                return None
        else:
            return None
        node = trie.advance(0, sm.buf)
        if node is None:
            return None
        ok = [i for i, t in enumerate(self.texts[:vocab_size]) if trie.token_valid(t, node)]
        return ok or None

    def mask_bits(self, vocab_size):
        import numpy as np
        w = (vocab_size + 63) // 64
        ok = self.allowed(vocab_size)
        if ok is None:
            return np.full(w, 0xFFFFFFFFFFFFFFFF, np.uint64), False
        bits = np.zeros(w, np.uint64)
        for i in ok:
            bits[i >> 6] |= np.uint64(1 << (i & 63))
        return bits, True


def encoder_input(vocab, query, tools_json, max_enc):
    """run_impl's encoder input (engine.rs:231-266), or [] for an empty run."""
    tools = parse_tools_json(tools_json)
    compact = compact_json(normalize_tools_json(tools_json, tools))
    q, t = vocab.encode(query), vocab.encode(compact)
    if (not q and not t) or max_enc == 0:
        return [], tools
    q_len = min(len(q), max(max_enc - 2, 0))
    rem = max(max_enc - (q_len + 1), 0)
    t_len = min(len(t), rem)
    return q[:q_len] + [TOOLS] + t[:t_len], tools
