"""The synthetic scenario generator: BASELINE shapes, a correct factorisation
(checked with scipy), determinism, and geometry shared across climates."""
import hashlib

import numpy as np
import pytest
import scipy.sparse as sp
import scipy.sparse.linalg as spla

from sbb_read import Blob


@pytest.fixture(scope="module")
def c1(built, tmp_path_factory):
    from neurips2026_smart_building_challenge_b200 import preset, write_scenario

    return write_scenario(tmp_path_factory.mktemp("g") / "c1.sbb", preset(1, 0))


def test_config1_shape(c1):
    b = Blob(c1)
    assert list(b.get("grid")) == [64, 48]
    assert len(b.get("solved")) == 3072
    assert len(b.get("zone_area")) == 41 and b.get("ahu_const").shape == (1, 9)
    assert list(b.get("sensed_shape")) == [41, 3072]
    assert len(b.get("weather_ambient")) == 8641 and b.get("obs_meta")[3] == 8640
    assert int(b.get("n_dev")[0]) == 6 * 41 + 10 + 7 and int(b.get("n_aux")[0]) == 7
    disc = b.get("act_is_discrete")
    assert (disc == 0).sum() == 2 * 41 + 3 + 2 and (disc == 1).sum() == 2


@pytest.mark.parametrize("index", [0, 14, 29])
def test_config2_shapes(built, tmp_path, index):
    from neurips2026_smart_building_challenge_b200 import preset, write_scenario

    rooms = [41, 49, 57, 65, 73, 81][index // 5]
    ahus = [1, 2, 2, 3, 3, 4][index // 5]
    b = Blob(write_scenario(tmp_path / "s.sbb", preset(2, index)))
    assert list(b.get("grid")) == [64, 48]
    assert len(b.get("zone_area")) == rooms and b.get("ahu_const").shape == (ahus, 9)
    amb = b.get("weather_ambient") - 273.15
    mean = [-5.0, 5.0, 15.0, 25.0, 32.0][index % 5]
    assert abs(amb.mean() - mean) < 1.5


def test_factor_reproduces_matrix(c1):
    b = Blob(c1)
    A = b.csc("A_system").tocsr()
    L, U = b.csc("lu_L"), b.csc("lu_U")
    pr, pc = b.get("lu_perm_r"), b.get("lu_perm_c")
    n = A.shape[0]
    # SuperLU convention: Pr A Pc = L U with (Pr A Pc)[i, j] = A[inv(pr)[i], inv(pc)[j]]
    ir = np.empty(n, np.int64)
    ir[pr] = np.arange(n)
    ic = np.empty(n, np.int64)
    ic[pc] = np.arange(n)
    B = A[ir][:, ic]
    diff = (L @ U - B).tocoo()
    assert np.abs(diff.data).max() <= 1e-10 * np.abs(A.data).max()
    assert (sp.tril(L, -1) != 0).nnz + n == L.nnz and np.allclose(L.diagonal(), 1.0)
    assert sp.tril(U, -1).nnz == 0


def test_solref_matches_scipy(c1):
    b = Blob(c1)
    A = b.csc("A_system")
    x_ref = spla.spsolve(A, b.get("solref_b"))
    x = b.get("solref_x")
    assert np.abs(x - x_ref).max() <= 1e-10 * np.abs(x_ref).max()
    assert np.abs(A @ x - b.get("solref_b")).max() <= 1e-10


def test_generator_is_deterministic(built, tmp_path):
    from neurips2026_smart_building_challenge_b200 import preset, write_scenario

    h = [hashlib.sha256(write_scenario(tmp_path / f"{i}.sbb", preset(2, 7)).read_bytes()).hexdigest()
         for i in range(2)]
    assert h[0] == h[1]


def test_climates_share_geometry(built, tmp_path):
    from neurips2026_smart_building_challenge_b200 import preset, write_scenario

    a = Blob(write_scenario(tmp_path / "a.sbb", preset(2, 10)))
    c = Blob(write_scenario(tmp_path / "c.sbb", preset(2, 13)))
    for name in ["lu_L_data", "lu_U_data", "lu_perm_r", "applied_data", "room_cells", "conv_cand_idx"]:
        assert np.array_equal(a.get(name), c.get(name)), name
    assert not np.array_equal(a.get("weather_ambient"), c.get("weather_ambient"))


def test_impossible_layout_is_an_error(built, tmp_path):
    from neurips2026_smart_building_challenge_b200 import preset, write_scenario

    with pytest.raises(RuntimeError, match="too small"):
        write_scenario(tmp_path / "x.sbb", preset(1, 0, rows=8, cols=8, n_rooms=60))
