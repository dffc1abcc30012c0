"""The token cache format (cdl_b200.data): build, split, reopen, append with a
tail, crash recovery, the meta file's keys, the loader's order and widening."""

import json

import numpy as np
import pytest
import torch

from cdl_b200.data import CACHE_FORMAT, DeviceBlockLoader, TokenCache, build_from_tokens

# the keys of cdl's meta.json (cdl/dataset/token_cache.py CacheMeta)
META_KEYS = {"format", "model_id", "tokenizer", "tokenizer_revision", "eos_token_id", "seq_len", "dtype", "ratios",
             "seed", "num_test_blocks", "num_calib_blocks", "n_train_blocks", "n_test_blocks", "tail",
             "docs_consumed"}


def _stream(n, hi=49152, seed=0):
    return np.random.default_rng(seed).integers(0, hi, n).astype(np.int64)


def test_build_split_and_reopen(tmp_path):
    seq, ntest = 16, 3
    toks = _stream(16 * 12 + 5)
    c = build_from_tokens(tmp_path, toks, seq_len=seq, num_test_blocks=ntest, num_calib_blocks=2,
                          model_id="m", tokenizer="t", eos_token_id=0, ratios={"web": 1.0}, seed=7)
    meta = json.loads((tmp_path / "meta.json").read_text())
    assert set(meta) == META_KEYS and meta["format"] == CACHE_FORMAT and meta["dtype"] == "uint16"
    assert c.n_train_blocks == 9 and len(c.test_dataset) == 3
    raw = np.fromfile(tmp_path / "tokens.u16", dtype=np.uint16)
    assert raw.size == 12 * seq
    # test blocks (the stream's last whole blocks) first, then the train blocks
    assert np.array_equal(raw[: 3 * seq], toks[9 * seq: 12 * seq])
    assert np.array_equal(raw[3 * seq:], toks[: 9 * seq])
    assert torch.equal(c.train_dataset[4], torch.from_numpy(toks[4 * seq: 5 * seq]))
    assert c.train_dataset[0].dtype == torch.int64
    assert torch.equal(c.calib_blocks(2), torch.from_numpy(toks[: 2 * seq].reshape(2, seq)))
    d = TokenCache.open(tmp_path, expect={"seq_len": seq, "seed": 7})
    assert d.n_train_blocks == 9
    with pytest.raises(ValueError):
        TokenCache.open(tmp_path, expect={"seq_len": 32})


def test_append_keeps_tail_and_recovers_from_a_crash(tmp_path):
    seq = 8
    toks = _stream(8 * 6)
    c = build_from_tokens(tmp_path, toks, seq_len=seq, num_test_blocks=1)
    more = _stream(20, seed=1)
    c.append_tokens(more, docs_consumed={"web": 3})
    assert c.n_train_blocks == 5 + 2 and c.meta.tail == more[16:].tolist()
    assert c.meta.docs_consumed == {"web": 3}
    c.append_tokens(_stream(4, seed=2))
    assert c.n_train_blocks == 8 and c.meta.tail == []
    assert torch.equal(c.train_dataset[6], torch.from_numpy(more[8:16]))
    assert torch.equal(c.train_dataset[7], torch.from_numpy(np.concatenate([more[16:], _stream(4, seed=2)])))
    # bytes written past the committed blocks (a crash before the meta write) are cut off on open
    with open(tmp_path / "tokens.u16", "ab") as f:
        f.write(b"\x01\x02\x03\x04")
    d = TokenCache.open(tmp_path)
    assert (tmp_path / "tokens.u16").stat().st_size == (1 + 8) * seq * 2 and d.n_train_blocks == 8
    with open(tmp_path / "tokens.u16", "r+b") as f:
        f.truncate(10)
    with pytest.raises(ValueError):
        TokenCache.open(tmp_path)


def test_wide_vocabulary_is_uint32(tmp_path):
    toks = _stream(4 * 10, hi=100000)
    c = build_from_tokens(tmp_path, toks, seq_len=4, num_test_blocks=2)
    assert c.meta.dtype == "uint32"
    batches = list(DeviceBlockLoader(c.train_dataset, 4, "cpu", shuffle=False))
    assert len(batches) == 2 and torch.equal(batches[0].reshape(-1), torch.from_numpy(toks[:16]))


def test_loader_order_is_the_dataloaders(tmp_path):
    """Same batches, in the same order, as torch's DataLoader(shuffle=True,
    drop_last=True) from the same global seed (how cdl's training loop
    draws them), over two epochs."""
    c = build_from_tokens(tmp_path, _stream(32 * 23), seq_len=32, num_test_blocks=2)
    torch.manual_seed(5)
    dl = torch.utils.data.DataLoader(c.train_dataset, 4, shuffle=True, drop_last=True)
    want = [b.clone() for _ in range(2) for b in dl]
    torch.manual_seed(5)
    loader = DeviceBlockLoader(c.train_dataset, 4, "cpu")
    got = [b.clone() for _ in range(2) for b in loader]
    assert len(got) == len(want) == 10
    for a, b in zip(got, want):
        assert a.dtype == torch.int64 and torch.equal(a, b)


@pytest.mark.gpu
def test_device_loader_on_cuda(tmp_path):
    c = build_from_tokens(tmp_path, _stream(64 * 40), seq_len=64, num_test_blocks=4)
    torch.manual_seed(1)
    want = [b.clone() for b in torch.utils.data.DataLoader(c.train_dataset, 8, shuffle=True, drop_last=True)]
    torch.manual_seed(1)
    got = [b.cpu() for b in DeviceBlockLoader(c.train_dataset, 8, "cuda")]
    assert len(got) == len(want) and all(torch.equal(a, b) for a, b in zip(got, want))
