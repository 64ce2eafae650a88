"""The fp32 DiT oracle itself: layout positions, RoPE tables and the timestep
sinusoid follow the reference's definitions, and the fp32 forward agrees with
an fp64 run of the same weights (the oracle adds no error of its own at the
end-to-end bar's scale)."""
import numpy as np
import torch

import dit_fixtures as fx
from oracle import oracle as O
from oracle import dit_ref as R
from mingproj import dit_forward as DF


def test_positions_keep_padded_offsets():
    # src/ming-layout.cc:19-60: image axis-0 = roundup32(cap_len) + 1; caption row i -> i + 1
    pos = R.positions(2, 3, 101)
    assert (pos[:6, 0] == 129).all()
    assert pos[:6, 1].tolist() == [0, 0, 0, 1, 1, 1] and pos[:6, 2].tolist() == [0, 1, 2] * 2
    assert pos[6:, 0].tolist() == list(range(1, 102)) and (pos[6:, 1:] == 0).all()
    assert np.array_equal(pos, DF.layout_positions(2, 3, 101))


def test_rope_table_matches_definition():
    pos = R.positions(4, 4, 37)
    c, s = R.rope_tables(pos, 128)
    # pair 16 is axis 1's first pair (freq 1), pair 40 is axis 2's first pair
    assert np.allclose(c[:16, 16], np.cos(pos[:16, 1].astype(np.float64)))
    assert np.allclose(s[:16, 40], np.sin(pos[:16, 2].astype(np.float64)))
    # pair 1 of axis 0: freq 256^(-2/32)
    assert np.allclose(c[:, 1], np.cos(pos[:, 0] * 256.0 ** (-2.0 / 32)).astype(np.float32))
    c2, s2 = DF.rope_tables(pos, 128, (32, 48, 48), 256.0)
    assert np.array_equal(c, c2) and np.array_equal(s, s2)


def test_timestep_embedding_cos_first():
    e = R.timestep_embedding(0.7)
    t = 300.0
    assert abs(e[0] - np.cos(t)) < 1e-6 and abs(e[128] - np.sin(t)) < 1e-6
    f1 = np.exp(-np.log(10000.0) / 128)
    assert abs(e[1] - np.cos(t * f1)) < 1e-6


def test_fp32_oracle_matches_fp64():
    torch.set_num_threads(max(1, torch.get_num_threads()))
    w = fx.as_f32(fx.make_weights(0))
    lat, cap, q, gh, gw = fx.make_inputs("case_c")
    args = (fx.DIM, fx.HEADS, fx.NREF, fx.NLAY, fx.CAPF)
    y32 = R.DitRef(w, *args).forward(fx.bf16_bits_to_f32(lat), fx.bf16_bits_to_f32(cap), q, gh, gw,
                                     fx.SIGMA).numpy()
    y64 = R.DitRef(w, *args, dtype=torch.float64).forward(
        fx.bf16_bits_to_f32(lat), fx.bf16_bits_to_f32(cap), q, gh, gw, fx.SIGMA).numpy()
    assert y32.shape == (gh * gw, fx.PATCH)
    assert O.rel_l2(y32, y64) < 1e-4
