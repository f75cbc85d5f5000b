"""nvkv_decode_advance (device-side decode-step metadata) against the
oracle's restatement of ModelRunner::prepare_model_input
(engine/model_runner.rs:69-160) on the same sequences: bit-exact positions,
slot_mapping, cu_seqlens_q/k and context lengths, over several consecutive
steps, for batches larger than one 1024-thread chunk."""
import numpy as np
import pytest
import torch

import nvkv
import nvkv_oracle as O
from nvkv import ops

pytestmark = pytest.mark.gpu


def _state(B, P, steps, seed):
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 3000, B).astype(np.int64)
    width = int((lens.max() + steps + P - 1) // P)  # pages appended ahead of the steps
    nblocks = B * width + 7
    perm = rng.permutation(nblocks).astype(np.int32)
    bt = perm[:B * width].reshape(B, width)
    return lens, bt, nblocks


def _bufs(B):
    dev = "cuda"
    return (torch.empty(B, dtype=torch.int64, device=dev), torch.empty(B, dtype=torch.int64,
            device=dev), torch.empty(B + 1, dtype=torch.int32, device=dev),
            torch.empty(B + 1, dtype=torch.int32, device=dev))


def _oracle_step(lens, bt, P):
    """The decode step whose last token makes each sequence lens[b] long: the
    runner's Sequence holds exactly the pages its tokens occupy."""
    seqs = [O.Seq(token_ids=[0] * int(L), block_table=[int(x) for x in bt[b, :(L + P - 1) // P]],
                  num_cached_tokens=int(L) - 1, num_new_tokens=1, block_size=P)
            for b, L in enumerate(lens)]
    _, pos, ctx = O.prepare_model_input(seqs, P)
    return pos, ctx


@pytest.mark.parametrize("B", [1, 257, 1500])
def test_decode_advance_matches_prepare_model_input(B):
    P, steps = 256, 4
    lens, bt, nblocks = _state(B, P, steps, B)
    seq_lens = torch.from_numpy(lens - 1).cuda()  # before the first step's token
    bt_dev = torch.from_numpy(bt).cuda()
    pos, slots, cuq, cuk = _bufs(B)
    cur = lens.copy()
    for _ in range(steps):
        ops.decode_advance(seq_lens, bt_dev, nblocks, P, pos, slots, cuq, cuk)
        torch.cuda.synchronize()
        opos, ctx = _oracle_step(cur, bt, P)
        assert np.array_equal(pos.cpu().numpy(), opos)
        assert np.array_equal(slots.cpu().numpy(), ctx.slot_mapping)
        assert np.array_equal(cuq.cpu().numpy().view(np.uint32), ctx.cu_seqlens_q)
        assert np.array_equal(cuk.cpu().numpy().view(np.uint32), ctx.cu_seqlens_k)
        assert np.array_equal(seq_lens.cpu().numpy(), ctx.context_lens)
        cur += 1
    assert nvkv.device_error() == 0


def test_decode_advance_missing_page_is_reported():
    """A sequence that grows into a page the table does not hold gets slot -1
    (the store skips it) and DEVERR_BLOCK_RANGE; the others are unaffected."""
    P = 256
    bt = torch.tensor([[3, 0], [5, 6]], dtype=torch.int32, device="cuda")
    seq_lens = torch.tensor([511, 100], dtype=torch.int64, device="cuda")  # seq 0 -> 512 fits
    pos, slots, cuq, cuk = _bufs(2)
    nvkv.device_error()
    ops.decode_advance(seq_lens, bt, 10, P, pos, slots, cuq, cuk)
    torch.cuda.synchronize()
    assert nvkv.device_error() == 0 and slots.tolist() == [0 * P + 255, 5 * P + 100]
    ops.decode_advance(seq_lens, bt, 10, P, pos, slots, cuq, cuk)  # seq 0 -> 513: page 2 missing
    torch.cuda.synchronize()
    assert nvkv.device_error() == nvkv._lib.DEVERR_BLOCK_RANGE
    assert slots.tolist() == [-1, 5 * P + 101] and pos.tolist() == [512, 101]
    assert cuk.tolist() == [0, 513, 615]


def test_decode_advance_in_a_graph():
    """Captured once, replayed: every replay is one more decode step."""
    P, B = 256, 64
    lens, bt, nblocks = _state(B, P, 6, 11)
    seq_lens = torch.from_numpy(lens - 1).cuda()
    bt_dev = torch.from_numpy(bt).cuda()
    pos, slots, cuq, cuk = _bufs(B)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.decode_advance(seq_lens, bt_dev, nblocks, P, pos, slots, cuq, cuk)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.decode_advance(seq_lens, bt_dev, nblocks, P, pos, slots, cuq, cuk)
    for _ in range(4):
        graph.replay()
    torch.cuda.synchronize()
    final = lens + 4  # warm-up call + 4 replays (the capture itself runs nothing)
    opos, ctx = _oracle_step(final, bt, P)
    assert np.array_equal(seq_lens.cpu().numpy(), final)
    assert np.array_equal(slots.cpu().numpy(), ctx.slot_mapping)
    assert np.array_equal(cuk.cpu().numpy().view(np.uint32), ctx.cu_seqlens_k)
    graph.reset()
