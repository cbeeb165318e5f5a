"""Fuel I/O on the CPU: the native safetensors reader (round trips, interoperability
with the `safetensors` package, fail-closed on corrupt files) and the byte-level BPE
tokenizer against the `tokenizers` library on tokenizer.json files it trained.

Mirrors the reference's loader / tokenizer unit tests
(engines/glm5-moe-nvfp4-2b/tests/test_safetensors.cc, test_tokenizer.cc).
"""
import json
import os
import random
import struct

import pytest
import torch

from rocket_b200.config import load_fuel
from rocket_b200.fuel import safetensors_io as sio
from rocket_b200.models import init_fuel_tensors


def test_fuel_round_trip_sharded(tmp_path):
    cfg = load_fuel("tiny-moe").model
    t = {k: v for k, v in init_fuel_tensors(cfg, 0).items() if not k.startswith("master.")}
    sio.save_dir(t, str(tmp_path), shard_bytes=1 << 20, meta={"fuel": "tiny-moe"})
    files = [f for f in os.listdir(tmp_path) if f.endswith(".safetensors")]
    assert len(files) > 1
    back = sio.load_dir(str(tmp_path))
    assert set(back) == set(t)
    for k in t:
        assert back[k].dtype == t[k].dtype and back[k].shape == t[k].shape, k
        assert torch.equal(back[k].reshape(-1).view(torch.uint8), t[k].contiguous().reshape(-1).view(torch.uint8)), k
    assert sio.metadata(os.path.join(tmp_path, files[0]))["fuel"] == "tiny-moe"


def test_interop_with_safetensors_package(tmp_path):
    st = pytest.importorskip("safetensors.torch")
    g = torch.Generator().manual_seed(0)
    t = {"a": torch.randn(3, 5, generator=g).bfloat16(), "b": torch.randint(0, 255, (7,), dtype=torch.uint8),
         "c": torch.randn(2, 2, 2, generator=g), "s": torch.tensor(1.5), "e": torch.empty(0, 4),
         "f8": torch.randn(4, 4, generator=g).to(torch.float8_e4m3fn), "i": torch.arange(6, dtype=torch.int64)}
    p1 = str(tmp_path / "theirs.safetensors")
    st.save_file(t, p1, metadata={"k": "v"})
    mine = sio.load_file(p1)
    for k in t:
        assert mine[k].dtype == t[k].dtype and mine[k].shape == t[k].shape
        assert torch.equal(mine[k].reshape(-1).view(torch.uint8), t[k].reshape(-1).view(torch.uint8))
    p2 = str(tmp_path / "mine.safetensors")
    sio.save_file(t, p2, {"k": "v"})
    theirs = st.load_file(p2)
    for k in t:
        assert theirs[k].dtype == t[k].dtype and theirs[k].shape == t[k].shape
        assert torch.equal(theirs[k].reshape(-1).view(torch.uint8), t[k].reshape(-1).view(torch.uint8))


def _write_raw(path, header: dict, data: bytes):
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + data)


@pytest.mark.parametrize("case", ["truncated", "outside", "size", "overlap", "dtype", "json"])
def test_reader_refuses_corrupt_files(tmp_path, case):
    p = str(tmp_path / "bad.safetensors")
    ok = {"x": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}
    if case == "truncated":
        _write_raw(p, ok, b"\0" * 4)
    elif case == "outside":
        _write_raw(p, {"x": {"dtype": "F32", "shape": [2], "data_offsets": [8, 16]}}, b"\0" * 8)
    elif case == "size":
        _write_raw(p, {"x": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8)
    elif case == "overlap":
        _write_raw(p, {"x": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
                       "y": {"dtype": "F32", "shape": [1], "data_offsets": [4, 8]}}, b"\0" * 8)
    elif case == "dtype":
        _write_raw(p, {"x": {"dtype": "Q4", "shape": [2], "data_offsets": [0, 8]}}, b"\0" * 8)
    else:
        with open(p, "wb") as f:
            h = b'{"x": {"dtype": "F32", '
            f.write(struct.pack("<Q", len(h)) + h + b"\0" * 8)
    with pytest.raises(Exception):
        sio.load_file(p)


# ---------------------------------------------------------------- tokenizer
def _corpus(n=400, seed=0):
    rnd = random.Random(seed)
    words = ["def", "return", "self", "import", "torch", "the", "of", "and", "kernel", "tensor", "函数", "über",
             "naïve", "😀", "x1", "42", "3.14", "foo_bar", "(", ")", ":", "    ", "\n", "\t", "'s", "'ll"]
    return [" ".join(rnd.choice(words) for _ in range(rnd.randint(3, 20))) for _ in range(n)]


def _train(pre_tokenizer, tmp_path, name, special=("<|endoftext|>", "<|user|>")):
    tk = pytest.importorskip("tokenizers")
    from tokenizers import decoders, models, trainers
    tok = tk.Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizer
    tok.decoder = decoders.ByteLevel()
    tr = trainers.BpeTrainer(vocab_size=600, special_tokens=list(special),
                             initial_alphabet=tk.pre_tokenizers.ByteLevel.alphabet())
    tok.train_from_iterator(_corpus(), trainer=tr)
    p = str(tmp_path / f"{name}.json")
    tok.save(p)
    return tok, p


def _check(tok, path):
    from rocket_b200.fuel.tokenizer import Tokenizer
    mine = Tokenizer.from_file(path)
    tests = _corpus(60, seed=1) + ["", " ", "   leading", "trailing   ", "a\n\n  b", "x<|endoftext|>y",
                                   "<|user|> hi 12345 6.5", "ñandú 😀😀 函数", "tabs\tand\r\nnewlines"]
    for s in tests:
        ref = tok.encode(s).ids
        got = mine.encode(s)
        assert got == ref, (s, got, ref)
        assert mine.decode(got) == tok.decode(ref, skip_special_tokens=False) or mine.decode(got) == s


def test_tokenizer_matches_tokenizers_bytelevel(tmp_path):
    tk = pytest.importorskip("tokenizers")
    tok, p = _train(tk.pre_tokenizers.ByteLevel(add_prefix_space=False), tmp_path, "gpt2style")
    _check(tok, p)


def test_tokenizer_matches_tokenizers_split_regex(tmp_path):
    """Qwen / GLM style: a Split regex with Unicode classes, then ByteLevel without its own regex."""
    tk = pytest.importorskip("tokenizers")
    pat = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*|"
           r"\s*[\r\n]+|\s+(?!\S)|\s+")
    pre = tk.pre_tokenizers.Sequence([
        tk.pre_tokenizers.Split(tk.Regex(pat), behavior="isolated"),
        tk.pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    tok, p = _train(pre, tmp_path, "qwenstyle")
    _check(tok, p)
