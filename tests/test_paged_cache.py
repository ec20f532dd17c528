"""Host logic of PagedKVCache (CPU tensors): same contract as the reference's
allocator (fskernels/paged_attn/paged_kv_cache.py:85-154)."""
import pytest
import torch

from fasterkernels_b200.paged_attn import PAGE_SIZE, PagedKVCache
from fasterkernels_b200 import workloads as W


def make(pages=8, seqs=3, blocks=4):
    return PagedKVCache(num_layers=2, num_pages=pages, max_seqs=seqs, max_blocks_per_seq=blocks, num_kv_heads=2,
                        head_dim=128, dtype=torch.float16, device="cpu")


def test_append_and_block_table():
    c = make()
    s = c.allocate_sequence()
    toks = []
    for i in range(PAGE_SIZE + 3):
        k = torch.full((1, 2, 1, 128), float(i), dtype=torch.float16)
        c.append_kv(s, 1, k, -k)
        toks.append(i)
    assert c.seq_len(s) == PAGE_SIZE + 3
    bt = c.get_block_table_tensor([s])
    assert bt.shape == (1, 4) and (bt[0, :2] >= 0).all() and (bt[0, 2:] == -1).all()
    p1 = int(bt[0, 1])
    assert float(c.k_pool[1, p1, 0, 2, 0]) == PAGE_SIZE + 2
    assert float(c.v_pool[1, p1, 1, 2, 5]) == -(PAGE_SIZE + 2)
    assert c.get_seq_lens_tensor([s]).tolist() == [PAGE_SIZE + 3]
    assert c.pages_used == 2 and c.pages_free == 6


def test_free_returns_pages_and_slots():
    c = make()
    a, b = c.allocate_sequence(), c.allocate_sequence()
    for _ in range(40):
        c.append_kv(a, 0, torch.zeros(1, 2, 1, 128, dtype=torch.float16), torch.zeros(1, 2, 1, 128, dtype=torch.float16))
    assert c.pages_used == 3
    c.free_sequence(a)
    assert c.pages_used == 0 and (c.block_table[a] == -1).all()
    assert c.allocate_sequence() == a
    c.allocate_sequence()
    with pytest.raises(RuntimeError, match="occupied"):
        c.allocate_sequence()
    assert "PagedKVCache" in repr(c)


def test_out_of_pages():
    c = make(pages=1)
    s = c.allocate_sequence()
    z = torch.zeros(1, 2, 1, 128, dtype=torch.float16)
    for _ in range(PAGE_SIZE):
        c.append_kv(s, 0, z, z)
    with pytest.raises(RuntimeError, match="Out of KV pages"):
        c.append_kv(s, 0, z, z)


def test_varlen_to_paged_roundtrip_cpu():
    lens = [1, 16, 17, 40]
    d = W.make_varlen(lens, 8, 2, torch.float16, "cpu", seed=3, sinks=False)
    kp, vp, bt = W.varlen_to_paged(d["k"], d["v"], lens, 1.25, seed=3)
    cu = d["cu_seqlens"]
    for b, L in enumerate(lens):
        for tok in range(L):
            p, o = divmod(tok, PAGE_SIZE)
            assert torch.equal(kp[int(bt[b, p]), :, o], d["k"][cu[b] + tok])
    assert len(set(bt[bt >= 0].tolist())) == sum((L + 15) // 16 for L in lens)


def test_config_lengths_match_the_seed_protocol():
    assert sum(W.config_lengths(2)) == 377152
    l3 = W.config_lengths(3)
    assert sum(l3) == 275479 and sum((L + 15) // 16 for L in l3) == 17244
    assert W.config_lengths(4) == [32768] * 16
    assert W.kv_bytes(W.config_lengths(2), 8, 2) == 1544814592


def test_lpt_partition_balances():
    lens = W.config_lengths(5)
    for n in (2, 4, 8):
        parts = W.lpt_partition(lens, n)
        assert sorted(i for p in parts for i in p) == list(range(len(lens)))
        loads = [sum(lens[i] for i in p) for p in parts]
        assert max(loads) / (sum(lens) / n) < 1.002


def test_begin_end_step_host_bookkeeping():
    c = make(pages=8, seqs=3, blocks=4)
    a, b = c.allocate_sequence(), c.allocate_sequence()
    z = torch.zeros(1, 2, 1, 128, dtype=torch.float16)
    for _ in range(15):
        c.append_kv(a, 0, z, z)
    bt, pos, lens = c.begin_step([a, b])
    # a (15 tokens) still fits its first page; b (0 tokens) gets a new page
    assert pos.tolist() == [15, 0] and lens.tolist() == [16, 1]
    assert c.pages_used == 2 and int(c.block_table[b, 0]) >= 0
    assert bt.shape == (2, 4) and bt[0, 0] == c.block_table[a, 0]
    new_lens = c.end_step()
    assert new_lens.tolist() == [16, 1] and c.seq_len(a) == 16
    c.begin_step([a])  # a crosses into its second page
    assert c.pages_used == 3 and int(c.block_table[a, 1]) >= 0


def test_write_prefill_pages_and_reserve():
    # the prompt of one layer lands token by token in its pages; reserve
    # pre-allocates the pages later decode steps will use
    c = PagedKVCache(num_layers=2, num_pages=20, max_seqs=2, max_blocks_per_seq=8, num_kv_heads=2, head_dim=4,
                     dtype=torch.float32, device="cpu")
    s = c.allocate_sequence()
    k = torch.randn(2, 37, 4)
    v = torch.randn(2, 37, 4)
    c.write_prefill(s, 1, k, v, reserve=60)
    assert c.seq_len(s) == 37
    bt = c.get_block_table_tensor([s])[0]
    assert (bt[:4] >= 0).all() and (bt[4:] == -1).all()  # ceil(60 / 16) pages
    pages = bt[:3].tolist()
    got_k = torch.cat([c.k_pool[1][p] for p in pages], dim=1)[:, :37]
    got_v = torch.cat([c.v_pool[1][p] for p in pages], dim=1)[:, :37]
    assert torch.equal(got_k, k) and torch.equal(got_v, v)
    assert float(c.k_pool[0].abs().sum()) == 0.0  # other layers untouched
    c.write_prefill(s, 0, k, v)  # the same prompt for layer 0: no new pages
    assert c.get_block_table_tensor([s])[0].tolist() == bt.tolist() and c.seq_len(s) == 37
    with pytest.raises(RuntimeError):
        c.write_prefill(s, 0, torch.zeros(2, 200, 4), torch.zeros(2, 200, 4))  # > max_blocks_per_seq
