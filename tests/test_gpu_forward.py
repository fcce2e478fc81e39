"""The batched device forward (mp_forward) vs the C oracle of CpuRunner::append.

Logits tolerance is the north star's: |gpu - oracle| <= 1e-3 + 1e-4 |oracle|,
and the greedy token (first maximum) must be identical.
"""
import numpy as np
import pytest

from oracle.oracle import Oracle
from tinyinfer_b200.synthetic import ModelConfig, random_tokens, random_weights

MINI = ModelConfig(layers=2, intermediate=128, vocabulary=256, context=64, tied=False)


def close(gpu, ref):
    err = np.abs(gpu - ref)
    assert (err <= 1e-3 + 1e-4 * np.abs(ref)).all(), f"max abs err {err.max():.3e}"
    assert int(np.argmax(gpu)) == int(np.argmax(ref))
    return float(err.max())


def device_for(config, weights, block_tokens, max_blocks, **kw):
    from tinyinfer_b200.device import DeviceContext

    ctx = DeviceContext(config, block_tokens=block_tokens, max_blocks=max_blocks, **kw)
    ctx.load_weights(weights)
    return ctx


@pytest.mark.gpu
def test_mini_prefill_then_decode(built):
    w = random_weights(MINI, seed=21)
    bt = 4
    ctx = device_for(MINI, w, bt, 32, max_sequences=4, max_step_tokens=64, max_step_sequences=4)
    o = Oracle(MINI, w, bt)
    keys, values = o.new_pools(32)
    blocks = [7, 3, 30, 12, 5, 9, 11, 2]
    ctx.table_write(2, 0, blocks)
    toks = random_tokens(20, MINI.vocabulary, 4)
    used = 0
    errs = []
    for chunk in (toks[:7], toks[7:8], toks[8:9], toks[9:16], toks[16:17]):
        t, f, lg, rc = ctx.forward([(2, used, len(chunk))], chunk)
        assert rc == 0 and f.all()
        ref, ok = o.append(keys, values, blocks, used, chunk)
        errs.append(close(lg[0], ref))
        assert t[0] == int(np.argmax(ref))
        used += len(chunk)
    print("mini max abs err", max(errs))
    ctx.close()


@pytest.mark.gpu
def test_mini_batched_equals_sequential(built):
    """Three sequences in one forward (prefill and decode mixed) give each sequence
    the oracle's logits; a row's result does not depend on its batch."""
    w = random_weights(MINI, seed=22)
    bt = 4
    ctx = device_for(MINI, w, bt, 64, max_sequences=8, max_step_tokens=64, max_step_sequences=8)
    o = Oracle(MINI, w, bt)
    pools = {s: o.new_pools(64) for s in range(3)}
    tables = {0: [1, 2, 3, 4, 5], 1: [10, 11, 12, 13, 14], 2: [20, 21, 22, 23, 24]}
    for s, b in tables.items():
        ctx.table_write(s, 0, b)
    rng = np.random.default_rng(3)
    prompts = {0: rng.integers(0, 256, 9), 1: rng.integers(0, 256, 1), 2: rng.integers(0, 256, 4)}
    used = {s: 0 for s in range(3)}
    # step 1: all prefill
    seqs = [(s, 0, len(prompts[s])) for s in range(3)]
    t, f, lg, rc = ctx.forward(seqs, np.concatenate([prompts[s] for s in range(3)]))
    assert rc == 0
    for s in range(3):
        ref, _ = o.append(*pools[s], tables[s], 0, prompts[s])
        close(lg[s], ref)
        used[s] = len(prompts[s])
    # steps 2..4: mixed decode and short prefill
    for step in range(3):
        chunks = {0: [int(t[0])], 1: list(rng.integers(0, 256, 2)), 2: [int(t[2])]}
        seqs = [(s, used[s], len(chunks[s])) for s in range(3)]
        t, f, lg, rc = ctx.forward(seqs, np.concatenate([chunks[s] for s in range(3)]))
        assert rc == 0
        for s in range(3):
            ref, _ = o.append(*pools[s], tables[s], used[s], chunks[s])
            close(lg[s], ref)
            used[s] += len(chunks[s])
    ctx.close()


@pytest.mark.gpu
def test_nonfinite_logits_reported(built):
    from tinyinfer_b200 import device

    w = random_weights(MINI, seed=23)
    w["model.embed_tokens.weight"][15, :] = np.nan
    ctx = device_for(MINI, w, 4, 16, max_sequences=2, max_step_tokens=16, max_step_sequences=2)
    ctx.table_write(0, 0, [0, 1])
    ctx.table_write(1, 0, [2, 3])
    t, f, lg, rc = ctx.forward([(0, 0, 2), (1, 0, 3)], [3, 15, 1, 2, 4])
    assert rc == device.MP_ERR_NONFINITE
    assert not f[0] and f[1]
    ctx.close()


@pytest.mark.gpu
def test_cow_region_copies_both_pools(built):
    """A merged TailCopyRegion (kv_manager.cpp:217-226) copies `width` floats of
    every layer row in both pools and nothing else (the payload check of
    miniprefix/tests/cow_test.cpp:57-117)."""
    ctx = device_for(MINI, random_weights(MINI, seed=1), 4, 8, max_sequences=2, max_step_tokens=8,
                     max_step_sequences=2)
    kvw, layers, bt = MINI.kv_width, MINI.layers, 4
    _, _, n = ctx.pools()
    keys = np.arange(1, n + 1, dtype=np.float32)
    ctx.kv_write(0, 0, keys)
    ctx.kv_write(1, 0, -keys)
    pitch = bt * kvw
    src, dst, valid = 2, 5, 3
    region = (dst * layers * pitch, src * layers * pitch, pitch, valid * kvw, layers)
    ctx.cow_copy([region])
    ctx.sync()
    k = ctx.kv_read(0, 0, n)
    v = ctx.kv_read(1, 0, n)
    expect = keys.copy()
    for row in range(layers):
        s0, d0 = region[1] + row * pitch, region[0] + row * pitch
        expect[d0:d0 + valid * kvw] = keys[s0:s0 + valid * kvw]
    assert np.array_equal(k, expect)
    assert np.array_equal(v, -expect)
    ctx.close()


def apply_regions(pool, regions):
    """Reference-layout effect of tail-copy regions applied as one step: every
    source read, then every destination written (in region order)."""
    out = pool.copy()
    rows = [[pool[s + r * p:s + r * p + w].copy() for r in range(n)] for d, s, p, w, n in regions]
    for (d, s, p, w, n), data in zip(regions, rows):
        for r in range(n):
            out[d + r * p:d + r * p + w] = data[r]
    return out


@pytest.mark.gpu
def test_pool_offsets_are_reference_layout(built):
    """The context's pools are layer-major on the device while mp_kv_read /
    mp_kv_write and COW regions take reference-layout element offsets
    ([block][layer][slot][192], miniprefix/include/miniprefix/paged_kv.h:25-27):
    ranges that start and end inside pages round-trip, and regions whose rows
    cross page boundaries (direct, and two-phase through a forward) copy exactly
    the elements they name."""
    ctx = device_for(MINI, random_weights(MINI, seed=3), 4, 8, max_sequences=2, max_step_tokens=8,
                     max_step_sequences=2)
    kvw, layers, bt = MINI.kv_width, MINI.layers, 4
    _, _, n = ctx.pools()
    page = bt * kvw
    block = layers * page
    assert n == 8 * block
    rng = np.random.default_rng(5)
    keys = rng.standard_normal(n).astype(np.float32)
    ctx.kv_write(0, 0, keys)
    ctx.kv_write(1, 0, -keys)
    for off, cnt in [(0, n), (4, 100), (page - 8, 24), (block - 4, block + 8), (3 * page + 12, n - 3 * page - 12),
                     (2 * block, 3 * block), (n - 4, 4)]:
        assert np.array_equal(ctx.kv_read(0, off, cnt), keys[off:off + cnt]), (off, cnt)
        assert np.array_equal(ctx.kv_read(1, off, cnt), -keys[off:off + cnt]), (off, cnt)
    patch = rng.standard_normal(2 * page + 40).astype(np.float32)
    at = page + 20
    ctx.kv_write(0, at, patch)
    ctx.kv_write(1, at, -patch)
    keys[at:at + patch.size] = patch
    assert np.array_equal(ctx.kv_read(0, 0, n), keys)
    assert np.array_equal(ctx.kv_read(1, 0, n), -keys)
    # direct copy: rows of 800 floats starting 16 floats before a page end
    direct = [(5 * block + 8, block + page - 16, 2 * page, page + 32, 2)]
    ctx.cow_copy(direct)
    ctx.sync()
    keys = apply_regions(keys, direct)
    assert np.array_equal(ctx.kv_read(0, 0, n), keys)
    assert np.array_equal(ctx.kv_read(1, 0, n), -keys)
    # two-phase: the second region's source overlaps the first one's destination
    chained = [(4 * block + 40, 2 * block + 700, block, 200, 2), (6 * block + 4, 4 * block + 100, block, 900, 2)]
    ctx.table_write(0, 0, [0])
    ctx.forward([(0, 0, 1)], [3], regions=chained, logits=False)
    keys = apply_regions(keys, chained)
    # block 0 holds the step's own K/V row
    assert np.array_equal(ctx.kv_read(0, block, n - block), keys[block:])
    assert np.array_equal(ctx.kv_read(1, block, n - block), -keys[block:])
    ctx.close()


@pytest.mark.gpu
def test_forward_cow_chain_reads_sources_first(built):
    """The COW regions of one batched step apply as if every source were read
    before any destination is written: with per-step publishing, the page a decode
    append copies away from is freed and handed to the next append's copy in the
    same step (page 4 below is both a source and a destination), so each
    destination must get its source's content from before the step."""
    ctx = device_for(MINI, random_weights(MINI, seed=2), 4, 12, max_sequences=2, max_step_tokens=8,
                     max_step_sequences=2)
    kvw, layers, bt = MINI.kv_width, MINI.layers, 4
    _, _, n = ctx.pools()
    keys = np.arange(1, n + 1, dtype=np.float32)
    ctx.kv_write(0, 0, keys)
    ctx.kv_write(1, 0, -keys)
    pitch = bt * kvw
    page = layers * pitch
    # (destination, source, valid rows): 3 <- 4, 4 <- 5, 5 <- 6, 6 <- 7 and an
    # independent 10 <- 9
    chain = [(3, 4, 3), (4, 5, 2), (5, 6, 1), (6, 7, 3), (10, 9, 2)]
    regions = [(d * page, s * page, pitch, v * kvw, layers) for d, s, v in chain]
    ctx.table_write(0, 0, [0])
    ctx.forward([(0, 0, 1)], [3], regions=regions, logits=False)
    k = ctx.kv_read(0, 0, n)
    v = ctx.kv_read(1, 0, n)
    expect = keys.copy()
    for d, s, rows in chain:
        for row in range(layers):
            s0, d0 = s * page + row * pitch, d * page + row * pitch
            expect[d0:d0 + rows * kvw] = keys[s0:s0 + rows * kvw]
    # page 0 holds the step's own K/V row; everything else must match exactly
    assert np.array_equal(k[page:], expect[page:])
    assert np.array_equal(v[page:], -expect[page:])
    ctx.close()


@pytest.mark.gpu
def test_135m_config1_prefix_and_greedy(built):
    """BASELINE config 1 shape (30 layers, vocab 49152, tied, page 16), shortened to a
    64-token prompt and 6 greedy steps so the C oracle finishes in seconds."""
    c = ModelConfig()
    w = random_weights(c, seed=1234)
    ctx = device_for(c, w, 16, 64, max_sequences=2, max_step_tokens=128, max_step_sequences=2)
    o = Oracle(c, w, 16)
    keys, values = o.new_pools(64)
    blocks = list(range(63, 40, -1))
    ctx.table_write(0, 0, blocks)
    prompt = random_tokens(64, c.vocabulary, 99)
    t, f, lg, rc = ctx.forward([(0, 0, 64)], prompt)
    ref, _ = o.append(keys, values, blocks, 0, prompt)
    errs = [close(lg[0], ref)]
    used, tok = 64, int(t[0])
    for _ in range(6):
        t, f, lg, rc = ctx.forward([(0, used, 1)], [tok])
        ref, _ = o.append(keys, values, blocks, used, [tok])
        errs.append(close(lg[0], ref))
        assert int(t[0]) == int(np.argmax(ref))
        used, tok = used + 1, int(t[0])
    print("135M max abs err", max(errs))
    ctx.close()
