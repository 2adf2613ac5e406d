"""Text front end of needle_run (C++ tokenizer, tool-JSON handling and
constrained-decoding masks, through the C ABI) against the reference restated
in Python (oracle/text_oracle.py) and the reference's own unit-test vectors:
to_snake_case cases (crates/needle-infer/src/tokenizer.rs:395-403) and the
trie / state machine / tool parsing / name mask cases
(crates/needle-infer/src/constrained.rs:693-779).  CPU only.

The token-id vectors of tokenizer.rs:305-392 need weights/vocab.txt, which is
not in this repository; the BPE algorithm is checked against the restatement
on a synthetic SentencePiece-style vocabulary instead."""
import numpy as np
import pytest

import text_oracle as to
from conftest import load_pkg

nb = load_pkg()
wl = load_pkg("needle_workload", "workload.py")

VOCAB_TEXT = wl.random_vocab(8192, 0)


@pytest.fixture(scope="module")
def vocabs():
    return nb.Vocab(VOCAB_TEXT), to.Vocab(VOCAB_TEXT)


def _random_text(rng):
    words = ["What", "is", "the", "weather", "in", "Paris", "get_weather", "New", "York", "book", "a", "flight",
             '{"name":"get_weather"}', "tutorials", "online", "café", "naïve", "中文", "🙂", "x=1,y=2", "(ok)",
             "tab\there", "UPPER", "snake_case", "dash-name", "3.14", "", "   "]
    seps = [" ", "  ", "\t", "\n", " ", "　", " ", "", " \r\n "]
    parts = []
    for _ in range(int(rng.integers(1, 12))):
        parts.append(words[int(rng.integers(len(words)))])
        parts.append(seps[int(rng.integers(len(seps)))])
    return "".join(parts)


# ── tokenizer ──────────────────────────────────────────────────────────────

def test_encode_matches_reference(vocabs):
    v, ref = vocabs
    rng = np.random.default_rng(0)
    for _ in range(400):
        t = _random_text(rng)
        assert v.encode(t) == ref.encode(t), repr(t)


@pytest.mark.parametrize("text", ["", " ", "\t\n\r", "　 ", "a", "🙂", "中", "a　　b",
                                  " leading and trailing ", "é" * 40, "x" * 300, '[{"name":"a","arguments":{}}]'])
def test_encode_edge_cases(vocabs, text):
    v, ref = vocabs
    assert v.encode(text) == ref.encode(text)


def test_decode_matches_reference(vocabs):
    v, ref = vocabs
    rng = np.random.default_rng(1)
    for _ in range(200):
        ids = rng.integers(0, 8192 + 20, int(rng.integers(0, 30))).tolist()  # ids past the vocab are skipped
        assert v.decode(ids) == ref.decode_ids(ids)
    t = "get weather information"
    assert v.decode(v.encode(t)) == t


def test_greedy_legacy_vocab():
    # a vocabulary file without scores encodes by greedy longest match
    legacy = "".join(line.split("\t")[0] + "\n" for line in VOCAB_TEXT.splitlines())
    v, ref = nb.Vocab(legacy), to.Vocab(legacy)
    rng = np.random.default_rng(2)
    for _ in range(200):
        t = _random_text(rng)
        assert v.encode(t) == ref.encode(t), repr(t)


def test_vocab_parse_quirks():
    # "\r\n" endings, a repeated piece (its last line wins), odd score fields
    text = ("<pad>\t0\r\n</s>\t0\n<s>\t0\n<unk>\t0\n<tool_call>\t0\n<tools>\t0\n▁\t0\na\t0\nb\t0\n"
            "ab\t-1\nab\t-2\n▁a\tinf\nba\tNaN\n▁ab\tgarbage\nbb\t-0.5e1\naa\t+3\r")
    v, ref = nb.Vocab(text), to.Vocab(text)
    assert len(v) == len(ref.id_to_piece)
    for t in ["ab", "a b", "abab", "bb aa", "ba ab", "aab", "  ab  ba "]:
        assert v.encode(t) == ref.encode(t), t


def test_bpe_ties_pick_the_leftmost_pair():
    # "ab" has one score; in "abab" both pairs score equally: the leftmost merges first
    text = "<pad>\t0\n</s>\t0\n<s>\t0\n<unk>\t0\n<tool_call>\t0\n<tools>\t0\n▁\t0\na\t0\nb\t0\nab\t-1\nbab\t-1\n"
    v, ref = nb.Vocab(text), to.Vocab(text)
    for t in ["abab", "babab", "ababab", "bab"]:
        assert v.encode(t) == ref.encode(t), t


# ── tool names and tool JSON ───────────────────────────────────────────────

def test_snake_case_reference_cases():
    cases = {"getWeather": "get_weather", "GetWeather": "get_weather", "get-weather": "get_weather",
             "get.weather": "get_weather", "HTMLParser": "html_parser", "already_snake": "already_snake"}
    for name, want in cases.items():
        assert nb.snake_case(name) == want == to.to_snake_case(name)


def test_snake_case_random():
    rng = np.random.default_rng(3)
    alphabet = list("aBcDxYZ09_-. ") + ["é"]
    for _ in range(500):
        name = "".join(rng.choice(alphabet, int(rng.integers(0, 14))))
        assert nb.snake_case(name) == to.to_snake_case(name), repr(name)


TOOLS = [
    '[{"name":"get_weather","description":"Get weather","parameters":{"location":{"type":"string"},'
    '"unit":{"type":"string"}}}]',
    '[{"name":"get_weather","parameters":{"type":"object","properties":{"location":{"type":"string"},'
    '"unit":{"type":"string"}},"required":["location"]}}]',
    '[{"name":"getWeather","parameters":{"city":{"type":"string"}}},'
    ' {"name":"sendEmail","description":"Send \\"mail\\" now","parameters":{"to":{},"body":{"type":"string"}}}]',
    '[ {"name": "spacedName", "parameters": {"a": {}}} ,\n  {"name":"HTMLParser","parameters":{}} ]',
    '{"name":"single.tool","parameters":{"x":{"nested":{"y":1}},"z":3}}',
    '[{"name":"unicodeTool","description":"naïve café 中文","parameters":{"clé":{}}}]',
    "no json at all",
    "",
]


@pytest.mark.parametrize("tools", TOOLS)
def test_tools_encoder_text_matches_reference(tools):
    defs = to.parse_tools_json(tools)
    assert nb.tools_encoder_text(tools) == to.compact_json(to.normalize_tools_json(tools, defs))


def test_parse_tools_reference_cases():
    flat = to.parse_tools_json(TOOLS[0])
    assert flat == [("get_weather", "get_weather", ["location", "unit"])]
    schema = to.parse_tools_json(TOOLS[1])
    assert schema[0][2] == ["location", "unit"]  # "type" / "required" excluded


@pytest.mark.parametrize("tools", TOOLS[:6])
def test_restore_tool_names_matches_reference(tools):
    defs = to.parse_tools_json(tools)
    for _, snake, keys in defs:
        out = '[{"name":"%s","arguments":{%s}}]' % (snake, ",".join('"%s":1' % k for k in keys))
        assert nb.restore_tool_names(tools, out) == to.restore_tool_names(out, defs)


# ── constrained decoding ───────────────────────────────────────────────────

def test_state_machine_reference_cases(vocabs):
    v, _ = vocabs
    c = nb.Constraint(TOOLS[0], v)
    c.feed(b'[{"name":"get_weather","arguments":{}}]')
    assert c.state == nb.Constraint.FREE
    c = nb.Constraint(TOOLS[0], v)
    c.feed(b'[{"name":"get_weather","arguments":{"')
    assert c.state == nb.Constraint.IN_ARG_KEY
    c = nb.Constraint(TOOLS[0], v)
    c.feed(b'[{"name":"get_weather","arguments":{"location":"Paris","unit":"celsius"}}]')
    assert c.state == nb.Constraint.FREE


def test_name_mask_reference_case():
    # constrained.rs:749-779: "get" allowed, " get" (space) and "set" blocked
    vocab = nb.Vocab("get\n▁get\nset\n")
    c = nb.Constraint('[{"name":"get_weather","parameters":{"location":{},"unit":{}}}]', vocab)
    c.feed(b'[{"name":"')
    assert c.state == nb.Constraint.IN_NAME
    bits, constrained = c.mask(3)
    assert constrained
    allowed = [(int(bits[0]) >> i) & 1 for i in range(3)]
    assert allowed == [1, 0, 0]


def test_masks_match_reference(vocabs):
    v, ref = vocabs
    V = 8192
    for tools in TOOLS[:6]:
        defs = to.parse_tools_json(tools)
        for _, snake, keys in defs or [("x", "x", [])]:
            out = '[{"name":"%s","arguments":{%s}}]' % (snake, ",".join('"%s":"v"' % k for k in keys))
            ob = out.encode()
            # byte by byte
            c, rc = nb.Constraint(tools, v), to.ConstrainedDecoder(defs, ref)
            for i in range(len(ob) + 1):
                bits, con = c.mask(V)
                rbits, rcon = rc.mask_bits(V)
                assert con == rcon and np.array_equal(bits, rbits), (tools, out[:i])
                if i < len(ob):
                    c.feed(ob[i:i + 1])
                    rc.sm.feed(ob[i:i + 1])
            # token by token, through the vocabulary's own pieces
            c, rc = nb.Constraint(tools, v), to.ConstrainedDecoder(defs, ref)
            for tok in ref.encode(out):
                bits, con = c.mask(V)
                rbits, rcon = rc.mask_bits(V)
                assert con == rcon and np.array_equal(bits, rbits)
                c.update(tok)
                rc.update(tok)


def test_text_entry_points_reject_bad_input():
    with pytest.raises(nb.NeedleError):
        nb.Vocab(b"\xff\xfe")
    assert not nb.lib().needle_snake_case(b"\xff\xfe")
    assert not nb.lib().needle_tools_encoder_text(b"[\xc0\xaf]")  # overlong UTF-8
