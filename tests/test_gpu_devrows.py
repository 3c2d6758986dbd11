"""Rows already in device memory (turbo_b200_embed_write_device): the plan is
built on the device and must be the host's entry for entry, so the vectors
equal a host write's bit for bit, with nothing but the sizes crossing PCIe."""
import numpy as np
import pytest

from turboembed_b200 import abi, models, runtime

pytestmark = pytest.mark.gpu

EXACT, FASTEST = abi.TURBO_PRECISION_EXACT, abi.TURBO_PRECISION_FASTEST


@pytest.fixture(scope="module")
def ctx():
    c = runtime.Backend().context(0)
    yield c
    c.release()


def awkward_rows(seed, batch, seq, vocab):
    """Varied lengths with ties, holes inside rows and left padding."""
    rng = np.random.default_rng(seed)
    ids = np.zeros((batch, seq), np.int32)
    mask = np.zeros((batch, seq), np.int32)
    for r in range(batch):
        n = int(rng.integers(1, seq + 1)) if r % 5 else seq // 2  # every fifth row the same length
        pad = int(rng.integers(0, 4)) if r % 3 == 0 else 0
        n = min(n, seq - pad)
        ids[r, pad:pad + n] = rng.integers(1000, vocab - 1, size=n)
        mask[r, pad:pad + n] = 1
        if n > 4 and r % 4 == 1:
            mask[r, pad + n // 2] = 0  # a hole
    types = (rng.random((batch, seq)) < 0.3).astype(np.int32)
    return ids, mask, types


@pytest.mark.parametrize("name,vocab,seq,precision", [("bert-base", 30522, 200, FASTEST), ("bert-base", 30522, 200, EXACT),
                                                      ("modernbert-base", 50368, 1500, FASTEST)])
def test_device_rows_give_the_host_writes_bits(ctx, name, vocab, seq, precision):
    import torch
    d = models.synthetic(name, 21, layers=2)
    batch = 23 if seq < 1000 else 3
    ids, mask, types = awkward_rows(33, batch, seq, vocab)
    if name == "modernbert-base":
        types = None
        mask[:, :1100] = 1  # long rows: the two-tile attention items too
    m = ctx.load(d)
    s = m.session(batch, seq, precision)
    dev = [torch.from_numpy(x).cuda() if x is not None else None for x in (ids, mask, types)]
    torch.cuda.synchronize()
    for pooling in (abi.TURBO_POOLING_MEAN, abi.TURBO_POOLING_CLS, abi.TURBO_POOLING_LAST):
        s.write(ids, mask, types, pooling=pooling)
        s.run()
        host = s.read().copy()
        s.write_device(dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr() if dev[2] is not None else 0, batch,
                       seq, pooling=pooling)
        run = s.run()
        assert run.h2d_bytes == 0
        got = s.read()
        assert np.isfinite(got).all()
        assert np.array_equal(got, host), (pooling, np.abs(got - host).max())
    s.release()
    m.release()


def test_device_rows_refuse_an_empty_row(ctx):
    import torch
    d = models.synthetic("minilm", 0, layers=1)
    ids = np.full((2, 16), 1000, np.int32)
    mask = np.ones((2, 16), np.int32)
    mask[1] = 0
    m = ctx.load(d)
    s = m.session(2, 16, FASTEST)
    di, dm = torch.from_numpy(ids).cuda(), torch.from_numpy(mask).cuda()
    with pytest.raises(runtime.TurboError) as e:
        s.write_device(di.data_ptr(), dm.data_ptr(), 0, 2, 16)
    assert e.value.code == abi.TURBO_E_INVALID_ARGUMENT
    s.release()
    m.release()


@pytest.mark.parametrize("bad", ["id_past_vocab", "negative_id", "type_past_types"])
def test_device_rows_refuse_ids_and_types_out_of_range(ctx, bad):
    # Host rows arrive checked by the core (core/src/session/tokens.rs:343);
    # device rows are checked on the device and refused by the host before
    # any run: the gather never reads past its tables.
    import torch
    d = models.synthetic("minilm", 0, layers=1)
    ids = np.full((3, 16), 1000, np.int32)
    mask = np.ones((3, 16), np.int32)
    types = np.zeros((3, 16), np.int32)
    if bad == "id_past_vocab":
        ids[2, 5] = 30522
    elif bad == "negative_id":
        ids[1, 0] = -1
    else:
        types[2, 3] = 2
    m = ctx.load(d)
    s = m.session(3, 16, FASTEST)
    di, dm, dt = (torch.from_numpy(x).cuda() for x in (ids, mask, types))
    torch.cuda.synchronize()
    with pytest.raises(runtime.TurboError) as e:
        s.write_device(di.data_ptr(), dm.data_ptr(), dt.data_ptr(), 3, 16)
    assert e.value.code == abi.TURBO_E_INVALID_ARGUMENT and "row" in e.value.message
    with pytest.raises(runtime.TurboError) as e:
        s.run()  # nothing was written
    assert e.value.code == abi.TURBO_E_INVALID_STATE
    # The same session takes good rows afterwards.
    ids[ids < 0] = 1000
    ids[ids >= 30522] = 1000
    types[:] = 0
    di, dt = torch.from_numpy(ids).cuda(), torch.from_numpy(types).cuda()
    torch.cuda.synchronize()
    s.write_device(di.data_ptr(), dm.data_ptr(), dt.data_ptr(), 3, 16)
    s.run()
    assert np.isfinite(s.read()).all()
    s.release()
    m.release()
