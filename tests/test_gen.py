"""CPU tests of the seeded generator (vrs_gen.cuh through the C ABI)."""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_philox_known_answers(tmp_path):
    # Random123 published known-answer vectors for Philox4x32-10.
    src = tmp_path / "kat.cpp"
    src.write_text(
        '#include "%s/vector-rs_b200/csrc/vrs_gen.cuh"\n#include <cstdio>\n'
        "int main(){auto p=[](vrs_gen::U4 c,uint32_t a,uint32_t b){auto r=vrs_gen::philox4x32_10(c,a,b);"
        'printf("%%08x%%08x%%08x%%08x\\n",r.x,r.y,r.z,r.w);};'
        "p({0,0,0,0},0,0);p({~0u,~0u,~0u,~0u},~0u,~0u);"
        "p({0x243f6a88u,0x85a308d3u,0x13198a2eu,0x03707344u},0xa4093822u,0x299f31d0u);}\n" % ROOT)
    exe = tmp_path / "kat"
    subprocess.run(["g++", "-std=c++17", "-O2", "-ffp-contract=off", str(src), "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    assert out == ["6627e8d5e169c58dbc57ac4c9b00dbd8", "408f276d41c83b0ea20bc7c66d5451fd",
                   "d16cfe0994fdcceb5001e42024126ea1"]


def test_rows_are_position_independent(vc):
    s = vc.config_seed(0)
    full = vc.gen_rows_host(vc.GEN_NORMAL, s, 0, 0, 64, 13)
    part = vc.gen_rows_host(vc.GEN_NORMAL, s, 0, 40, 24, 13)
    assert np.array_equal(full[40:], part)


def test_distributions(vc):
    z = vc.gen_rows_host(vc.GEN_NORMAL, vc.config_seed(0), 0, 0, 8000, 128).astype(np.float64)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1) < 0.01 and abs((z ** 4).mean() - 3) < 0.05
    u = vc.gen_rows_host(vc.GEN_NORMAL_UNIT, vc.config_seed(1), 0, 0, 100, 128)
    assert np.allclose(np.linalg.norm(u.astype(np.float64), axis=1), 1, atol=1e-6)
    w = vc.gen_rows_host(vc.GEN_UNIFORM, vc.config_seed(3), 0, 0, 1000, 96)
    assert w.min() >= 0 and w.max() < 1 and abs(w.mean() - 0.5) < 0.01
    h = vc.gen_rows_host(vc.GEN_UNIFORM_SUM1, vc.config_seed(3), 0, 0, 100, 96)
    assert np.allclose(h.astype(np.float64).sum(1), 1, atol=1e-5)
    c = vc.gen_rows_host(vc.GEN_NORMAL, vc.config_seed(2), 2, 0, 16, 8)
    m = vc.gen_rows_host(vc.GEN_MIXTURE, vc.config_seed(2), 0, 0, 4000, 8, c, 16, 0.1)
    # every point lies within a few sigma of one centre
    d = ((m[:, None, :] - c[None]) ** 2).sum(-1).min(1)
    assert d.max() < 8 * 0.1 ** 2 * 8
