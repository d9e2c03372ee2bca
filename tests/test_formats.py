"""Scene formats against files written by the reference's own exporter
(tests/golden/scene_v*.foam from scripts/export_for_viewer.py write_foam)."""
import os

import numpy as np
import pytest

from vorotracing_b200 import formats

GD = os.path.join(os.path.dirname(__file__), "golden")
IN = np.load(os.path.join(GD, "foam_inputs.npz"))


def _write(tmp_path, version, spec=True):
    p = tmp_path / f"out_v{version}.foam"
    pts = IN["points"]
    formats.write_foam(p, pts, IN["density"], IN["diffuse"], IN["specular"] if spec else None,
                       IN["adj"], IN["offs"], IN["poses"], 4, 4, 0.01, 1e-3, 512,
                       aabb=(pts.min(0), pts.max(0)), adjacent_diff=IN["adj_diff"],
                       version=version)
    return p


@pytest.mark.parametrize("version,spec,golden", [(4, True, "scene_v4.foam"),
                                                 (3, True, "scene_v3.foam"),
                                                 (4, False, "scene_v4_nospec.foam")])
def test_writer_matches_reference_bytes(tmp_path, version, spec, golden):
    ours = open(_write(tmp_path, version, spec), "rb").read()
    ref = open(os.path.join(GD, golden), "rb").read()
    assert ours == ref


@pytest.mark.parametrize("golden", ["scene_v4.foam", "scene_v3.foam", "scene_v4_nospec.foam"])
def test_reader_parses_reference_files(golden):
    d = formats.read_foam(os.path.join(GD, golden))
    np.testing.assert_array_equal(d["points"], IN["points"])
    np.testing.assert_array_equal(d["density"], IN["density"])
    np.testing.assert_array_equal(d["diffuse_h4"].view(np.uint16), IN["diffuse"].view(np.uint16))
    if d["has_specular"]:
        np.testing.assert_array_equal(d["specular_h4"].view(np.uint16),
                                      IN["specular"].view(np.uint16))
    else:
        assert not d["specular_h4"].any()
    np.testing.assert_array_equal(d["adj"], IN["adj"])
    np.testing.assert_array_equal(d["offs"], IN["offs"])
    np.testing.assert_array_equal(d["poses"], IN["poses"])
    np.testing.assert_array_equal(d["default_pose"], IN["poses"][0])
    assert d["max_intersections"] == 512 and abs(d["weight_threshold"] - 0.01) < 1e-9
    if d["version"] == 3:
        np.testing.assert_array_equal(d["adjacent_diff"].view(np.uint16),
                                      IN["adj_diff"].view(np.uint16))


def test_checkpoint_roundtrip(tmp_path):
    from vorotracing_b200 import scene as sc

    s = sc.make_scene(500, 3, False, 4, cache=False)
    p = tmp_path / "scene.pt"
    formats.save_checkpoint(p, s["points"], np.log(s["density"]), s["adj"], s["offs"],
                            s["diffuse"], s["specular"])
    d = formats.load_checkpoint(p)
    np.testing.assert_allclose(d["density"], s["density"], rtol=1e-6)
    for k in ("points", "adj", "offs", "diffuse", "specular"):
        np.testing.assert_array_equal(d[k], s[k])


def test_bad_magic(tmp_path):
    p = tmp_path / "bad.foam"
    p.write_bytes(b"\0" * 200)
    with pytest.raises(ValueError, match="not a .foam"):
        formats.read_foam(p)


def test_reads_reference_checkpoint():
    """A checkpoint written by the reference's VoroTracing.save_checkpoint."""
    import torch

    raw = torch.load(os.path.join(GD, "checkpoint_ref.pt"), map_location="cpu")
    d = formats.load_checkpoint(os.path.join(GD, "checkpoint_ref.pt"))
    np.testing.assert_array_equal(d["points"], raw["xyz"].numpy())
    np.testing.assert_allclose(d["density"], np.exp(raw["density"].numpy()), rtol=1e-6)
    np.testing.assert_array_equal(d["adj"], raw["adjacency"].numpy().astype(np.uint32))
    np.testing.assert_array_equal(d["offs"], raw["adjacency_offsets"].numpy().astype(np.uint32))
    assert d["diffuse"].shape == (16, 48) and d["specular"].shape == (16, 48)


def test_written_checkpoint_has_reference_keys(tmp_path):
    import torch

    ref = torch.load(os.path.join(GD, "checkpoint_ref.pt"), map_location="cpu")
    d = formats.load_checkpoint(os.path.join(GD, "checkpoint_ref.pt"))
    p = tmp_path / "again.pt"
    formats.save_checkpoint(p, d["points"], np.log(d["density"]), d["adj"], d["offs"],
                            d["diffuse"], d["specular"])
    ours = torch.load(p, map_location="cpu")
    assert set(ours) == set(ref)
    for k in ref:
        assert ours[k].dtype == ref[k].dtype and ours[k].shape == ref[k].shape, k
        torch.testing.assert_close(ours[k], ref[k], rtol=1e-6, atol=0)
