"""The batched data-parallel server (include/b2s_server.h): host logic on CPU with fake engines, and the
real BitVLA-shape engines on a B200.

The fakes are Python engines called from the server's C++ worker threads. They check that requests are
batched (up to max_batch per engine call), that every request gets its own observation's result, that a
failing engine's requests come back with that engine's status and message while the other engines keep
serving, and that a server with no healthy engine fails requests instead of hanging.
"""
import threading
import time

import numpy as np
import pytest

IMG, NT, NA = 48, 4, 6  # small observation shape for the fakes


def fake_actions(img, tok):
    """Deterministic per-observation result: a function of that observation's bytes only."""
    return np.concatenate([img.reshape(len(img), -1)[:, :3].astype(np.float32),
                           tok[:, :3].astype(np.float32)], axis=1)


class FakeEngine:
    def __init__(self, delay=0.0, fail=False):
        self.delay, self.fail = delay, fail
        self.batches = []

    def predict(self, img, tok):
        import b2s
        self.batches.append(len(img))
        time.sleep(self.delay)
        if self.fail:
            raise b2s.B2SError(b2s.B2S_ERR_CUDA, "fake engine lost its GPU")
        return fake_actions(img, tok)


def obs(i):
    g = np.random.Generator(np.random.PCG64(i))
    return g.integers(0, 256, IMG).astype(np.uint8), g.integers(0, 1000, NT).astype(np.int32)


def test_batches_and_results(b2s):
    from b2s.server import Server
    engines = [FakeEngine(delay=0.02), FakeEngine(delay=0.02)]
    srv = Server(engines, IMG, NT, NA, max_batch=4, queue_capacity=64)
    ids = [srv.submit(*obs(i)) for i in range(40)]
    used = set()
    for i, rid in enumerate(ids):
        act, lat, eng = srv.wait(rid)
        img, tok = obs(i)
        assert np.array_equal(act, fake_actions(img[None], tok[None])[0])
        assert lat >= 0.0 and eng in (0, 1)
        used.add(eng)
    assert used == {0, 1}                                 # both engines served
    assert max(max(e.batches) for e in engines) > 1       # requests were batched
    assert all(b <= 4 for e in engines for b in e.batches)
    st = srv.engine_status()
    assert sum(s["completed"] for s in st) == 40 and all(s["healthy"] for s in st)
    srv.close()


def test_failing_engine_others_keep_serving(b2s):
    from b2s.server import Server
    engines = [FakeEngine(delay=0.01), FakeEngine(delay=0.01, fail=True), FakeEngine(delay=0.01)]
    srv = Server(engines, IMG, NT, NA, max_batch=2, queue_capacity=64)
    ids = [srv.submit(*obs(i)) for i in range(30)]
    ok, failed = 0, 0
    for i, rid in enumerate(ids):
        try:
            act, _, eng = srv.wait(rid)
            img, tok = obs(i)
            assert eng != 1 and np.array_equal(act, fake_actions(img[None], tok[None])[0])
            ok += 1
        except b2s.B2SError as e:
            assert e.status == b2s.B2S_ERR_CUDA and "lost its GPU" in str(e) and e.engine == 1
            failed += 1
    st = srv.engine_status()
    assert not st[1]["healthy"] and st[0]["healthy"] and st[2]["healthy"]
    assert failed == st[1]["completed"] and 1 <= failed <= 2   # only the one batch it took
    assert ok == 30 - failed
    srv.close()


def test_no_healthy_engine_fails_fast(b2s):
    from b2s.server import ERR_UNAVAILABLE, Server
    srv = Server([FakeEngine(fail=True)], IMG, NT, NA, max_batch=1, queue_capacity=8)
    ids = [srv.submit(*obs(i)) for i in range(3)]
    statuses = []
    for rid in ids:
        with pytest.raises(b2s.B2SError) as ei:
            srv.wait(rid, timeout_ms=5000)
        statuses.append(ei.value.status)
    assert statuses[0] == b2s.B2S_ERR_CUDA
    assert all(s in (b2s.B2S_ERR_CUDA, ERR_UNAVAILABLE) for s in statuses)
    with pytest.raises(b2s.B2SError) as ei:
        srv.submit(*obs(9))
    assert ei.value.status == ERR_UNAVAILABLE
    srv.close()


def test_queue_bound_and_wait_timeout(b2s):
    from b2s.server import ERR_BUSY, ERR_TIMEOUT, Server
    gate = threading.Event()

    class Slow(FakeEngine):
        def predict(self, img, tok):
            gate.wait(10)
            return fake_actions(img, tok)

    srv = Server([Slow()], IMG, NT, NA, max_batch=1, queue_capacity=2)
    first = srv.submit(*obs(0))
    time.sleep(0.2)  # the worker takes it and blocks on the gate
    queued = [srv.submit(*obs(1)), srv.submit(*obs(2))]
    with pytest.raises(b2s.B2SError) as ei:
        srv.submit(*obs(3))
    assert ei.value.status == ERR_BUSY
    with pytest.raises(b2s.B2SError) as ei:
        srv.wait(first, timeout_ms=50)
    assert ei.value.status == ERR_TIMEOUT
    gate.set()
    for i, rid in enumerate([first] + queued):
        act, _, _ = srv.wait(rid)
        img, tok = obs(i)
        assert np.array_equal(act, fake_actions(img[None], tok[None])[0])
    srv.close()


def test_concurrent_clients(b2s):
    from b2s.server import Server
    srv = Server([FakeEngine(), FakeEngine()], IMG, NT, NA, max_batch=8, queue_capacity=512)
    errors = []

    def client(c):
        try:
            for k in range(25):
                i = 1000 * c + k
                act, _, _ = srv.wait(srv.submit(*obs(i)))
                img, tok = obs(i)
                assert np.array_equal(act, fake_actions(img[None], tok[None])[0])
        except Exception as e:  # pragma: no cover - reported below
            errors.append(e)

    th = [threading.Thread(target=client, args=(c,)) for c in range(6)]
    for t in th:
        t.start()
    for t in th:
        t.join(60)
    assert not errors
    assert sum(s["completed"] for s in srv.engine_status()) == 150
    srv.close()


@pytest.mark.gpu
def test_bitvla_server_matches_predict(b2s):
    """Real engines: every GPU of the box (at least one) serves reduced-depth BitVLA-shape observations; each
    request's actions equal b2s_bitvla_predict of the same observation alone, bit for bit."""
    import torch
    from b2s import bitvla
    from b2s.server import Server
    cfg = bitvla.default_config(vit_layers=2, dec_layers=2)
    devs = list(range(torch.cuda.device_count()))
    srv = Server.bitvla(devs, cfg, 4321, max_batch=4, queue_capacity=64)
    g = np.random.Generator(np.random.PCG64(3))
    n = 12
    imgs = g.integers(0, 256, (n, cfg.image_size, cfg.image_size, 3)).astype(np.uint8)
    toks = g.integers(0, cfg.vocab, (n, cfg.n_text)).astype(np.int32)
    ids = [srv.submit(imgs[i], toks[i]) for i in range(n)]
    got = [srv.wait(r)[0] for r in ids]
    srv.close()
    torch.cuda.set_device(0)
    m = bitvla.Model(cfg, 4321, max_batch=1)
    for i in range(n):
        ref = np.zeros((1, cfg.action_chunk * cfg.action_dim), np.float32)
        m.predict(imgs[i:i + 1], toks[i:i + 1], ref)
        assert np.array_equal(got[i], ref[0]), i
    m.close()
