"""CPU checks of bench.py's host-side pieces: the CPU baseline leg (the C
oracle's chain on all host cores and on one core, bounded samples) and the
seeded config-5 inputs the timed chain and its parity record share."""
import numpy as np


def test_cpu_baseline_record_all_cores_and_one_core():
    import bench
    from oracle import oracle as orc

    rec = bench.cpu_baseline_record(orc, 1024, 256, seconds=0.2, one_core_seconds=0.1)
    assert rec["kind"] == "port" and rec["unit"] == "GB/s"
    assert rec["cores"] >= 1 and rec["value"] > 0
    assert rec["one_core"]["cores"] == 1 and rec["one_core"]["value"] > 0
    # the oracle is left on every core for the legs that follow
    assert orc.num_threads() == rec["cores"]


def test_config5_inputs_are_seeded_and_shaped():
    import bench

    for C, aux_shape in ((1024, (1, 4096, 2)), (2048, (4096, 3))):
        a = bench.make_inputs(4096, C, 20261201, None)
        b = bench.make_inputs(4096, C, 20261201, None)
        assert a["x"].shape == (4096, C) and tuple(a["aux"].shape) == aux_shape
        assert np.array_equal(a["x"].float().numpy(), b["x"].float().numpy())
        # x ~ N(0, 1), shift / scale ~ N(0, 0.1)
        assert abs(float(a["x"].float().std()) - 1.0) < 0.01
        assert abs(float(a["shift"].float().std()) - 0.1) < 0.02
    c = bench.make_inputs(4096, 2048, 20261201, None)["aux"].numpy()
    assert c.min() == 0 and c.max() == 63  # voxel coordinates cycle over the 64^3 grid
