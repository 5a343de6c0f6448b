"""The output projection that feeds the sampler (model.nim:466-470 ->
matmul, model.nim:179-189): nls_lm_head against the CPU oracle.

CPU: the C restatement (oracle/ref_lmhead.c) equals the line-by-line Python
transliteration (oracle/translit.py) bit for bit on every weight type, both
paths (int8 activations, and dequantRow + dotF32) and batch sizes on either
side of the Q8_0 switch at nb = 4 (model.nim:185), including activation
blocks that are all zero, hold rounding ties or are all equal.

GPU: every logit equals the oracle's bit for bit (integer block products,
then the reference's fp32 operations in its order), on both tile layouts
(rows padded in shared memory when a row is a multiple of 16 bytes, one
contiguous copy otherwise), ragged row counts, batch tiles, and the
full-size Llama-3 shape (128256 x 4096).
"""
from __future__ import annotations

import numpy as np
import pytest

TYPES = {"f32": 0, "f16": 1, "q4_0": 2, "q8_0": 8, "q6_k": 14}


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _x(rng, nb, cols, edge=False):
    x = rng.standard_normal((nb, cols)).astype(np.float32)
    if edge and cols >= 64:
        x[0, :32] = 0.0                                    # amax = 0: d = 0, every q = 0
        x[-1, 32:64] = np.float32(0.25)                    # equal values: q = 127 each
        # values whose scaled v lands on k + 0.5 exactly (v + 0.5 rounding ties)
        x[0, 32:64] = np.float32(127.0) * np.linspace(-1, 1, 32, dtype=np.float32)
        x[0, 33] = np.float32(63.5)
    return x


def test_oracle_matches_transliteration(pkg, oracle_mod):
    from oracle import translit
    W = pkg.workloads
    rng = np.random.default_rng(11)
    for name, cols in [("f32", 75), ("f16", 64), ("q4_0", 96), ("q8_0", 64), ("q6_k", 256)]:
        t = TYPES[name]
        w = W.lm_weights(t, 5, cols, seed=5)
        if t == 8:  # a zero, a negative, a subnormal and an infinite... scale (finite ones only)
            w = w.copy()
            w[0, 0:2] = 0
            w[1, 0:2] = np.array([0x00, 0xA8], np.uint8)   # -2^-5
            w[2, 0:2] = np.array([0x01, 0x00], np.uint8)   # smallest subnormal half
        for nb in (1, 4, 5):
            x = _x(rng, nb, cols, edge=True)
            for exact in (False, True):
                got = oracle_mod.lm_head(w, t, 5, cols, x, exact_matmul=exact)
                want = np.array(translit.lm_head(w.reshape(-1), t, 5, cols, x, exact_matmul=exact),
                                dtype=np.float32)
                assert np.array_equal(_bits(got), _bits(want)), (name, nb, exact)


def test_quantize_act_known_answers(oracle_mod):
    # quantizeAct (quant.nim:646-662): d = amax/127, q = round half away from zero
    x = np.zeros(32, np.float32)
    d, q = oracle_mod.quantize_act(x, 32)
    assert d[0] == 0 and not q.any()
    x = np.arange(32, dtype=np.float32) - 16            # amax 16: id = 127/16 = 7.9375
    d, q = oracle_mod.quantize_act(x, 32)
    assert d[0] == np.float32(16) / np.float32(127)
    idv = np.float32(1) / d[0]
    want = [int(np.float32(v * idv) + np.float32(0.5)) if v * idv >= 0 else -int(-np.float32(v * idv) + np.float32(0.5))
            for v in x]
    assert q.tolist() == want and q[0] == -127


# ---- GPU parity ---------------------------------------------------------------

def _device_weights(w):
    import torch
    return torch.from_numpy(np.ascontiguousarray(w)).cuda()


def _check(engine, oracle_mod, w, t, rows, cols, x, exact, what):
    dw = _device_weights(w)
    got = engine.lm_head(dw, t, rows, cols, x, exact=exact)
    want = oracle_mod.lm_head(w, t, rows, cols, x, exact_matmul=exact, threads=16)
    bad = np.nonzero(_bits(got) != _bits(want))
    assert bad[0].size == 0, f"{what}: {bad[0].size} logits differ, first at {bad[0][0]},{bad[1][0]} " \
        f"gpu {got[bad[0][0], bad[1][0]]!r} oracle {want[bad[0][0], bad[1][0]]!r}"


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(TYPES))
@pytest.mark.parametrize("exact", [False, True])
def test_types_and_paths(pkg, engine, oracle_mod, name, exact):
    t = TYPES[name]
    rng = np.random.default_rng(t + 100 * exact)
    cols = 4096 if t != 0 else 1024
    rows = 3001
    w = pkg.workloads.lm_weights(t, rows, cols, seed=9)
    for nb in (1, 2, 4, 5, 9):
        x = _x(rng, nb, cols, edge=True)
        _check(engine, oracle_mod, w, t, rows, cols, x, exact, f"{name} nb={nb} exact={exact}")


@pytest.mark.gpu
@pytest.mark.parametrize("name,cols", [("q8_0", 96), ("q4_0", 160), ("q6_k", 768), ("f16", 100),
                                       ("f32", 4099), ("q8_0", 8192), ("q6_k", 3072),
                                       ("q8_0", 3584), ("q4_0", 3072), ("q8_0", 16384),
                                       ("q6_k", 2048), ("q6_k", 8192)])
def test_row_layouts(pkg, engine, oracle_mod, name, cols):
    """Rows that are not a multiple of 16 bytes (one contiguous copy per
    tile, the weights' last bytes by plain loads), a dotF32 tail (cols % 8),
    block counts that are not powers of two (idle term threads), and wide
    rows (few rows per tile; Q8_0 at 16384 columns takes the generic loop)."""
    t = TYPES[name]
    rng = np.random.default_rng(cols)
    rows = 777
    w = pkg.workloads.lm_weights(t, rows, cols, seed=2)
    for nb in (1, 3):
        for exact in (False, True):
            x = _x(rng, nb, cols)
            _check(engine, oracle_mod, w, t, rows, cols, x, exact, f"{name} cols={cols} nb={nb}")


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["q8_0", "q6_k"])
def test_llama3_output_layer(pkg, engine, oracle_mod, name):
    """The full Llama-3 output projection: 128256 x 4096, one decode row."""
    t = TYPES[name]
    rows, cols = 128256, 4096
    w = pkg.workloads.lm_weights(t, rows, cols, seed=1)
    x = np.random.default_rng(3).standard_normal((1, cols)).astype(np.float32)
    _check(engine, oracle_mod, w, t, rows, cols, x, False, f"{name} 128256x4096")


@pytest.mark.gpu
def test_device_tensors_and_status(pkg, engine, oracle_mod):
    import torch
    t, rows, cols = 8, 5000, 2048
    w = pkg.workloads.lm_weights(t, rows, cols, seed=4)
    dw = _device_weights(w)
    x = np.random.default_rng(5).standard_normal((3, cols)).astype(np.float32)
    got = engine.lm_head(dw, t, rows, cols, torch.from_numpy(x).cuda())
    want = oracle_mod.lm_head(w, t, rows, cols, x, threads=16)
    assert np.array_equal(_bits(got.cpu().numpy()), _bits(want))
    # weights uploaded through the library (nls_device_upload), host x and y
    wdev = engine.upload(w)
    try:
        assert wdev % 256 == 0
        assert np.array_equal(_bits(engine.lm_head(wdev, t, rows, cols, x)), _bits(want))
    finally:
        engine.free_device(wdev)
    # a non-finite activation on the int8 path is an error
    xb = x.copy()
    xb[1, 7] = np.inf
    _, st = None, None
    y = np.empty((3, rows), np.float32)
    lib = engine._lib
    import ctypes
    st = lib.nls_lm_head(engine._h, ctypes.c_void_p(dw.data_ptr()), t, rows, cols,
                         ctypes.c_void_p(xb.ctypes.data), 3, ctypes.c_void_p(y.ctypes.data), 0,
                         ctypes.c_void_p(0))
    assert st == 5
    # bad arguments: unaligned weights, an unknown type, cols not whole blocks
    for wp, tt, cc in [(dw.data_ptr() + 2, 8, cols), (dw.data_ptr(), 3, cols), (dw.data_ptr(), 8, 100)]:
        st = lib.nls_lm_head(engine._h, ctypes.c_void_p(wp), tt, rows, cc,
                             ctypes.c_void_p(x.ctypes.data), 1, ctypes.c_void_p(y.ctypes.data), 0,
                             ctypes.c_void_p(0))
        assert st == 1


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["q8_0", "q6_k", "f16"])
def test_lm_head_then_sample(pkg, big_engine_lm, oracle_mod, name):
    """nls_lm_head_sample: the projection's logits stay on the GPU and are
    sampled there; ids and probabilities equal the oracle's sampler run on
    the oracle's logits (config-3 sampling parameters, 64 rows)."""
    t = TYPES[name]
    V, cols, B = 32000, 2048, 64
    w = pkg.workloads.lm_weights(t, V, cols, seed=8, sigma=0.06)
    x = np.random.default_rng(9).standard_normal((B, cols)).astype(np.float32)
    s = pkg.workloads.make("c3_batched_hetero", seed=77, rows=np.arange(B), V=V)
    dw = _device_weights(w)
    ids, probs, st = big_engine_lm.lm_head_sample(
        dw, t, V, cols, x, s.params, s.hist_ids, s.hist_off, s.bias_ids, s.bias_vals, s.bias_off,
        s.uniforms, want_probs=True)
    assert st == 0
    logits = oracle_mod.lm_head(w, t, V, cols, x, threads=16)
    ref, dg = oracle_mod.sample_batch(logits, s.params, s.hist_ids, s.hist_off, s.bias_ids,
                                      s.bias_vals, s.bias_off, s.uniforms, threads=16, diag=True)
    bad = [int(i) for i in np.nonzero(ids != ref)[0] if dg["margin"][i] >= 1e-6]
    assert not bad, f"ids differ at rows {bad[:10]}"
    ok = (s.params["temperature"] > 0) & (ids == ref)
    rel = np.abs(probs[ok].astype(np.float64) - dg["prob"][ok]) / np.maximum(np.abs(dg["prob"][ok]), 1e-30)
    assert np.all(rel <= 1e-5)


@pytest.fixture(scope="module")
def big_engine_lm(pkg):
    eng = pkg.Engine(0, max_rows=256, max_vocab=1 << 17)
    yield eng
    eng.close()


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["q8_0", "q6_k"])
def test_row_slices_equal_whole(pkg, engine, name):
    """A tensor-parallel lm_head gives rank r the rows [r*Vs, (r+1)*Vs) of the
    output layer: projecting slices of the rows separately must give exactly
    the logits of the whole call (a row's dot product never depends on the
    other rows)."""
    import torch
    t, V, cols = TYPES[name], 6000, 4096
    w = pkg.workloads.lm_weights(t, V, cols, seed=21)
    dw = torch.from_numpy(w).cuda()
    x = np.random.default_rng(22).standard_normal((1, cols)).astype(np.float32)
    whole = engine.lm_head(dw, t, V, cols, x)
    parts = [engine.lm_head(dw[lo:hi], t, hi - lo, cols, x)
             for lo, hi in [(0, 2000), (2000, 4000), (4000, 6000)]]
    assert np.array_equal(whole.view(np.uint32), np.concatenate(parts, axis=1).view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["q8_0", "q4_0", "q6_k"])
def test_special_block_scales(pkg, engine, oracle_mod, name):
    """Block scales that are +inf, NaN, the smallest subnormal half and -0
    (a corrupt or extreme model file): the logits follow the same IEEE
    operations as the oracle's, bit for bit where they are numbers and NaN
    where its are (NaN payloads are not compared: x86 and the GPU quiet them
    differently)."""
    t = TYPES[name]
    rows, cols = 512, 1024
    w = pkg.workloads.lm_weights(t, rows, cols, seed=31).copy()
    bb = {8: 34, 2: 18, 14: 210}[t]
    off = {8: 0, 2: 0, 14: 208}[t]      # byte offset of the fp16 scale d in a block
    specials = [0x7C00, 0x7E00, 0x0001, 0x8000, 0xFC00]  # +inf, NaN, subnormal, -0, -inf
    for i, h in enumerate(specials):
        for r in range(i, rows, 37):
            blk = (r * 7 + i) % (w.shape[1] // bb)
            w[r, blk * bb + off] = h & 0xFF
            w[r, blk * bb + off + 1] = h >> 8
    x = np.random.default_rng(32).standard_normal((2, cols)).astype(np.float32)
    dw = _device_weights(w)
    for exact in (False, True):
        got = engine.lm_head(dw, t, rows, cols, x, exact=exact)
        want = oracle_mod.lm_head(w, t, rows, cols, x, exact_matmul=exact, threads=16)
        nan_g, nan_w = np.isnan(got), np.isnan(want)
        assert np.array_equal(nan_g, nan_w), f"{name} exact={exact}: NaN positions differ"
        assert nan_w.any()
        ok = ~nan_w
        assert np.array_equal(got[ok].view(np.uint32), want[ok].view(np.uint32)), f"{name} exact={exact}"


@pytest.mark.gpu
@pytest.mark.parametrize("cols,rows", [(256, 1000), (4096, 3001), (8192, 515)])
def test_q6_k_tensor_core_path(pkg, engine, oracle_mod, cols, rows):
    """Q6_K at 8 or more batch rows runs on the tensor cores: each block's
    16 sub-block sums from int8 MMAs, then the reference's scale products and
    fp32 terms in block order. Batch sizes below the switch (5), one and two
    16-row launches, a last launch of 8 rows (24) and tails of fewer than 8
    rows on the other path (17, 33); a partial last tile of 128 rows, one
    block per row (cols 256) and rows too wide for the tensor-core path's
    shared memory (cols 8192: the other path); activation blocks that are
    zero, equal or hold rounding ties."""
    t = TYPES["q6_k"]
    rng = np.random.default_rng(cols + rows)
    w = pkg.workloads.lm_weights(t, rows, cols, seed=cols)
    for nb in (5, 8, 16, 17, 24, 33):
        x = _x(rng, nb, cols, edge=True)
        _check(engine, oracle_mod, w, t, rows, cols, x, False, f"q6_k cols={cols} rows={rows} nb={nb}")


def _oracle_independent(oracle_mod, w, t, rows, cols, x):
    """Rows that are separate sequences: one-row matmuls (the int8 path for
    Q8_0 at any count); a call of at most 4 rows takes the same path and
    gives every row the same logits."""
    return np.concatenate([oracle_mod.lm_head(w, t, rows, cols, x[i:i + 4], threads=16)
                           for i in range(0, x.shape[0], 4)])


@pytest.mark.gpu
@pytest.mark.parametrize("cols,rows", [(256, 1000), (4096, 3001), (4352, 300), (8192, 515)])
def test_q8_0_tensor_core_path(pkg, engine, oracle_mod, cols, rows):
    """Q8_0 rows that are separate sequences (the int8 path at any count)
    run on the tensor cores from 8 rows: each block's sum from an int8 MMA,
    then (d_w * d_a) * float(s) in block order. Batch sizes below the switch
    (5), one and two 16-row launches, a last launch of 8 rows (24) and tails
    of fewer than 8 rows on the other path (17, 33); a partial last tile of
    128 rows, one 256-value step per row (cols 256), the widest row that
    fits the shared memory (4352) and one that does not (8192: the other
    path); activation blocks that are zero, equal or hold rounding ties."""
    t = TYPES["q8_0"]
    rng = np.random.default_rng(cols + rows + 1)
    w = pkg.workloads.lm_weights(t, rows, cols, seed=cols + 1)
    dw = _device_weights(w)
    for nb in (5, 8, 16, 17, 24, 33):
        x = _x(rng, nb, cols, edge=True)
        got = engine.lm_head(dw, t, rows, cols, x, independent=True)
        want = _oracle_independent(oracle_mod, w, t, rows, cols, x)
        bad = np.nonzero(_bits(got) != _bits(want))
        assert bad[0].size == 0, f"q8_0 cols={cols} nb={nb}: {bad[0].size} logits differ, first at " \
            f"{bad[0][0]},{bad[1][0]}"


@pytest.mark.gpu
@pytest.mark.parametrize("cols,rows", [(256, 1000), (4096, 3001), (6144, 300), (8192, 515)])
def test_q4_0_tensor_core_path(pkg, engine, oracle_mod, cols, rows):
    """Q4_0 (the int8 path at any batch size) on the tensor cores from 8
    rows: nibbles minus 8 as int8 operands, one MMA per block, then
    (d_w * d_a) * float(s) in block order; the same batch sizes and edges as
    Q8_0, 6144 the widest row that fits the shared memory."""
    t = TYPES["q4_0"]
    rng = np.random.default_rng(cols + rows + 2)
    w = pkg.workloads.lm_weights(t, rows, cols, seed=cols + 2)
    for nb in (5, 8, 16, 17, 24, 33):
        x = _x(rng, nb, cols, edge=True)
        _check(engine, oracle_mod, w, t, rows, cols, x, False, f"q4_0 cols={cols} rows={rows} nb={nb}")


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["q8_0", "q4_0", "q6_k"])
@pytest.mark.parametrize("rows", [1, 77])
def test_tensor_core_path_fewer_rows_than_a_tile(pkg, engine, oracle_mod, name, rows):
    """Weight matrices smaller than one 128-row tile (a single row too): the
    staged box reaches past the matrix (rows there read as zeros and are
    never stored), on both staging modes (Q6_K at 768 columns: rows of 630
    bytes, one bulk copy per row; the others: the tensor-map copy)."""
    t = TYPES[name]
    cols = 768
    w = pkg.workloads.lm_weights(t, rows, cols, seed=rows + t)
    x = _x(np.random.default_rng(rows + 3 * t), 9, cols, edge=True)
    got = engine.lm_head(_device_weights(w), t, rows, cols, x, independent=True)
    want = _oracle_independent(oracle_mod, w, t, rows, cols, x)
    assert np.array_equal(_bits(got), _bits(want)), f"{name} rows={rows}"


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["q8_0", "q4_0"])
def test_32_value_blocks_tensor_core_path_special_scales(pkg, engine, oracle_mod, name):
    """Block scales d that are +inf, NaN, subnormal, -0 and -inf, and
    blocks of extreme values (Q8_0: -128 and 127; Q4_0: nibbles 0 and 15)
    on the tensor-core path."""
    t = TYPES[name]
    bb = {"q8_0": 34, "q4_0": 18}[name]
    rows, cols = 640, 1024
    w = pkg.workloads.lm_weights(t, rows, cols, seed=43).copy()
    specials = [0x7C00, 0x7E00, 0x0001, 0x8000, 0xFC00]
    for i, h in enumerate(specials):
        for r in range(i, rows, 37):
            blk = (r * 7 + i) % (cols // 32)
            w[r, blk * bb] = h & 0xFF
            w[r, blk * bb + 1] = h >> 8
    w[::5, 2:bb] = 0x80 if name == "q8_0" else 0x00        # q = -128 / every nibble 0 (-8)
    w[1::5, bb + 2:2 * bb] = 0x7F if name == "q8_0" else 0xFF  # q = 127 / every nibble 15 (7)
    x = np.random.default_rng(44).standard_normal((11, cols)).astype(np.float32)
    got = engine.lm_head(_device_weights(w), t, rows, cols, x, independent=True)
    want = _oracle_independent(oracle_mod, w, t, rows, cols, x)
    nan_g, nan_w = np.isnan(got), np.isnan(want)
    assert np.array_equal(nan_g, nan_w)
    assert nan_w.any()
    ok = ~nan_w
    assert np.array_equal(got[ok].view(np.uint32), want[ok].view(np.uint32))
    # a non-finite activation on this path is an error, as on the others
    import ctypes
    xb = x.copy()
    xb[9, 700] = np.nan
    y = np.empty((11, rows), np.float32)
    dw = _device_weights(w)
    st = engine._lib.nls_lm_head(engine._h, ctypes.c_void_p(dw.data_ptr()), t, rows, cols,
                                 ctypes.c_void_p(xb.ctypes.data), 11, ctypes.c_void_p(y.ctypes.data),
                                 8, ctypes.c_void_p(0))
    assert st == 5


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["f16", "q8_0", "q4_0"])
def test_float_path_batch_tiles(pkg, engine, oracle_mod, name):
    """The float path (dequantRow + dotF32) tiled across batch rows: one,
    two and four batch rows per thread with padded batch groups (3, 7, 12),
    several 16-row launches (21, 33) and a partial last tile of rows; both
    the reference's own switch (Q8_0 above 4 rows) and exactMatmul."""
    t = TYPES[name]
    rng = np.random.default_rng(t + 7)
    rows, cols = 1000, 1024
    w = pkg.workloads.lm_weights(t, rows, cols, seed=t + 3)
    for nb in (2, 3, 7, 12, 16, 21, 33):
        x = _x(rng, nb, cols, edge=True)
        for exact in (False, True):
            _check(engine, oracle_mod, w, t, rows, cols, x, exact, f"{name} nb={nb} exact={exact}")


@pytest.mark.gpu
def test_q6_k_tensor_core_path_special_scales(pkg, engine, oracle_mod):
    """Block scales d that are +inf, NaN, subnormal, -0 and -inf, and
    extreme sub-block scales (-128, 127) on the tensor-core path."""
    t = TYPES["q6_k"]
    rows, cols = 640, 1024
    w = pkg.workloads.lm_weights(t, rows, cols, seed=41).copy()
    specials = [0x7C00, 0x7E00, 0x0001, 0x8000, 0xFC00]
    for i, h in enumerate(specials):
        for r in range(i, rows, 37):
            blk = (r * 7 + i) % 4
            w[r, blk * 210 + 208] = h & 0xFF
            w[r, blk * 210 + 209] = h >> 8
    w[::5, 192:208] = np.array([0x80, 0x7F] * 8, np.uint8)  # sub-block scales -128, 127
    w[::5, :128] = 0x00                                      # q = 0 (-32 after the offset)
    w[::5, 128:192] = 0x00
    x = np.random.default_rng(42).standard_normal((7, cols)).astype(np.float32)
    got = engine.lm_head(_device_weights(w), t, rows, cols, x, exact=False)
    want = oracle_mod.lm_head(w, t, rows, cols, x, exact_matmul=False, threads=16)
    nan_g, nan_w = np.isnan(got), np.isnan(want)
    assert np.array_equal(nan_g, nan_w)
    assert nan_w.any()
    ok = ~nan_w
    assert np.array_equal(got[ok].view(np.uint32), want[ok].view(np.uint32))


# ---- golden fixtures (tests/golden/make_golden_lmhead.py) ---------------------

def _golden_lmhead():
    import os
    z = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "lmhead_cases.npz"))
    return {k: z[k] for k in z.files}


def _golden_cases(g):
    for name, t in TYPES.items():
        for nb in (1, 5):
            for exact in (0, 1):
                yield name, t, nb, exact, g[f"w_{name}"], g["x"][:nb], g[f"y_{name}_{nb}_{exact}"]


def test_oracle_matches_golden(oracle_mod):
    g = _golden_lmhead()
    for name, t, nb, exact, w, x, y in _golden_cases(g):
        got = oracle_mod.lm_head(w, t, w.shape[0], x.shape[1], x, exact_matmul=bool(exact))
        assert np.array_equal(_bits(got), _bits(y)), (name, nb, exact)


@pytest.mark.gpu
def test_gpu_matches_golden(engine):
    g = _golden_lmhead()
    for name, t, nb, exact, w, x, y in _golden_cases(g):
        got = engine.lm_head(_device_weights(w), t, w.shape[0], x.shape[1], x, exact=bool(exact))
        assert np.array_equal(_bits(got), _bits(y)), (name, nb, exact)
