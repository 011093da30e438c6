"""The continuous-batching loop (inferox_b200/serving.py) on CPU against a
fake batch whose next token depends only on that sequence's own history:
every request, served among others with slots reused, must produce what
Model::generate (forward.rs:592-612) produces for it alone. The GPU side of
the calls it makes (prefill of one slot, a step over a subset of slots, a
slot reset) is held to the oracle in tests/test_gpu_batch.py."""
import numpy as np
import pytest

from inferox_b200.serving import Server, last_argmax

V = 97


def _next(history):
    h = 0
    for t in history:
        h = (h * 31 + int(t) + 7) % 1000003
    return h % V


class FakeBatch:
    def __init__(self, batch, max_seq):
        self.batch, self.max_seq = batch, max_seq
        self.hist = [[] for _ in range(batch)]
        self.prefills, self.resets, self.steps = [], [], 0

    def _grow(self, slot, toks):
        self.hist[slot].extend(int(t) for t in toks)
        if len(self.hist[slot]) > self.max_seq:
            raise RuntimeError("KV cache is full")

    def prefill(self, slot, ids, last_row_only=False):
        assert last_row_only
        self.prefills.append(slot)
        self._grow(slot, ids)
        want = _next(self.hist[slot])
        logits = np.zeros((1, V), np.float32)
        logits[0, want] = 5.0
        logits[0, (want * 3) % want if want else 0] = 5.0 if want else 0.0  # a tie below `want`
        return logits

    def decode_step_seqs(self, seqs, tokens, want_logits=True):
        assert len(set(seqs)) == len(seqs) and len(seqs) == len(tokens)
        self.steps += 1
        out = []
        for s, t in zip(seqs, tokens):
            self._grow(s, [t])
            out.append(_next(self.hist[s]))
        return None, np.array(out, np.uint32)

    def reset(self, slot):
        self.resets.append(slot)
        self.hist[slot] = []


def _alone(prompt, max_tokens, eos=None):
    """forward.rs:592-612 on a fresh single-sequence fake, stopping at eos."""
    fb = FakeBatch(1, 10_000)
    toks = [last_argmax(fb.prefill(0, prompt, True)[0])]
    while len(toks) < max_tokens and not (eos is not None and toks[-1] == eos):
        _, a = fb.decode_step_seqs([0], [toks[-1]])
        toks.append(int(a[0]))
    return toks


def test_last_argmax_ties():
    assert last_argmax([1, 3, 3, 0]) == 2
    assert last_argmax([2.0]) == 0


def test_requests_match_their_solo_runs():
    rng = np.random.default_rng(3)
    fb = FakeBatch(3, 40)
    srv = Server(fb)
    reqs = []
    for i in range(9):
        p = rng.integers(3, V, size=int(rng.integers(1, 8)))
        n = int(rng.integers(1, 12))
        eos = int(rng.integers(0, V)) if i % 3 == 0 else None
        reqs.append((srv.submit(p, n, eos), p, n, eos))
    srv.step()
    assert len(srv.waiting) == 6  # three slots filled first come, first served
    out = srv.run()
    for rid, p, n, eos in reqs:
        want = _alone(p, n, eos)
        assert out[rid] == want, (rid, out[rid], want)
        assert srv.result(rid) == want
    assert fb.prefills[:3] == [0, 1, 2] and len(fb.prefills) == 9
    assert sorted(set(fb.resets)) == [0, 1, 2]  # every slot was reused
    solo_steps = sum(len(_alone(p, n, e)) - 1 for _, p, n, e in reqs)
    assert srv.steps < solo_steps  # steps were shared between requests
    assert not srv.busy()


def test_limits():
    fb = FakeBatch(2, 10)
    srv = Server(fb)
    with pytest.raises(ValueError):
        srv.submit([], 3)
    with pytest.raises(ValueError):
        srv.submit([5], 0)
    with pytest.raises(ValueError):
        srv.submit(list(range(3, 9)), 6)  # 6 + 6 - 1 = 11 rows > 10
    rid = srv.submit(list(range(3, 8)), 6)  # 5 + 6 - 1 = 10 rows: fits exactly
    assert srv.result(rid) is None
    srv.run()
    assert len(srv.result(rid)) == 6 and len(fb.hist[0]) == 10
    one = srv.submit([4, 5], 1)  # finishes at admission, no decode step
    steps = srv.steps
    srv.run()
    assert srv.result(one) == _alone([4, 5], 1) and srv.steps == steps


def test_failed_prefill_keeps_the_request():
    """A prefill that raises (a CUDA or cache error) leaves the request
    waiting at the front; once the cause is gone it is served as if nothing
    had happened, in a slot that was reset first."""

    class Flaky(FakeBatch):
        fail = 1

        def prefill(self, slot, ids, last_row_only=False):
            if self.fail:
                self.fail -= 1
                self.hist[slot].extend([1, 2, 3])  # partial work left behind
                raise RuntimeError("device error")
            return super().prefill(slot, ids, last_row_only)

    fb = Flaky(2, 64)
    srv = Server(fb)
    prompt = [5, 9, 11]
    rid = srv.submit(prompt, 6)
    with pytest.raises(RuntimeError):
        srv.step()
    assert srv.result(rid) is None and len(srv.waiting) == 1
    while srv.busy():
        srv.step()
    assert srv.result(rid) == _alone(prompt, 6)
    assert fb.resets == [0]  # the slot the failed prefill touched was reset


class PoolEmpty(RuntimeError):
    name = "OutOfMemory"


class FakePaged(FakeBatch):
    """FakeBatch over a shared pool of `pages` pages of 4 rows: a call that
    needs more pages than are free raises the paged batch's OutOfMemory
    error and changes nothing, as ifx_kv_batch_create_paged's batch does."""

    ROWS = 4

    def __init__(self, batch, max_seq, pages):
        super().__init__(batch, max_seq)
        self.total = pages

    def pages(self):
        used = sum(-(-len(h) // self.ROWS) for h in self.hist)
        return self.total - used, self.total

    def _need(self, grow):
        extra = sum(-(-(len(self.hist[s]) + n) // self.ROWS) - -(-len(self.hist[s]) // self.ROWS)
                    for s, n in grow.items())
        if extra > self.pages()[0]:
            raise PoolEmpty("the page pool is exhausted")

    def prefill(self, slot, ids, last_row_only=False):
        self._need({slot: len(ids)})
        return super().prefill(slot, ids, last_row_only)

    def decode_step_seqs(self, seqs, tokens, want_logits=True):
        self._need({s: 1 for s in seqs})
        return super().decode_step_seqs(seqs, tokens, want_logits)


def test_paged_pool_preempts_and_requests_match_solo_runs():
    """Four slots over a pool that holds far fewer rows than four full
    requests: prefills wait for pages, decode steps preempt the youngest
    request, and every request still produces its solo tokens."""
    rng = np.random.default_rng(5)
    fb = FakePaged(4, 64, pages=9)  # 36 rows for 4 slots of up to 64
    srv = Server(fb)
    assert srv.paged
    reqs = []
    for i in range(10):
        p = rng.integers(3, V, size=int(rng.integers(2, 10)))
        n = int(rng.integers(4, 16))
        reqs.append((srv.submit(p, n), p, n))
    out = srv.run()
    for rid, p, n in reqs:
        assert out[rid] == _alone(p, n), rid
    assert srv.preemptions > 0
    assert fb.pages() == (9, 9)  # every page returned


def test_paged_pool_too_small_for_one_request():
    fb = FakePaged(2, 64, pages=2)
    srv = Server(fb)
    srv.submit(list(range(3, 12)), 4)  # 9 prompt rows need 3 pages
    with pytest.raises(PoolEmpty):
        srv.step()
    fb2 = FakePaged(2, 64, pages=2)
    srv2 = Server(fb2)
    srv2.submit([3, 4, 5], 12)  # fits at admission, outgrows the pool alone
    with pytest.raises(PoolEmpty):
        srv2.run()
