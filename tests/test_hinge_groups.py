"""The hinge-group schedule of the host model (zeno_b200/csrc/model.cpp, hinge_groups),
checked on the CPU for every bundled scene.

Both step kernels solve the colour-sorted joint constraints as groups (a hinge's point,
axis and angle-limit constraints on one body pair) and the general and two-lane kernels
run those groups by dependency level.  The result equals the reference's colour sweep
only if (1) every constraint appears exactly once, (2) each dynamic body sees its
constraints in sweep order, and (3) the groups of one level share no dynamic body.  A small
harness compiled from the product's own loader and model sources prints the schedule."""
import json
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "zeno_b200" / "csrc"

HARNESS = r'''
#include "model.h"
#include "scene.h"
#include <cstdio>
#include <fstream>
#include <sstream>
using namespace zb;
int main(int argc, char** argv) {
  std::ifstream f(argv[1]);
  std::stringstream ss;
  ss << f.rdbuf();
  Scene sc;
  std::string err;
  if (!load_mjcf(ss.str(), ".", &sc, &err, false)) { std::printf("{\"error\": \"load\"}\n"); return 1; }
  HostModel h;
  if (!build_model(sc, &h, &err)) { std::printf("{\"error\": \"model\"}\n"); return 1; }
  std::printf("{\"constraints\": [");
  for (size_t k = 0; k < h.constraints.size(); ++k)
    std::printf("%s[%u, %u, %u]", k ? ", " : "", h.constraints[k].body_a, h.constraints[k].body_b,
                h.constraints[k].type & 0xFFu);
  std::printf("], \"dynamic\": [");
  for (size_t b = 0; b < h.bodies.size(); ++b)
    std::printf("%s%d", b ? ", " : "", h.bodies[b].inv_mass_inertia[0] > 0.0f ? 1 : 0);
  std::printf("], \"groups\": [");
  for (size_t g = 0; g + 3 < h.hinge_groups.size(); g += 4)
    std::printf("%s[%u, %u, %u, %u]", g ? ", " : "", h.hinge_groups[g], h.hinge_groups[g + 1],
                h.hinge_groups[g + 2], h.hinge_groups[g + 3]);
  std::printf("], \"words\": [");
  for (size_t i = 0; i < h.jgroup_words.size(); ++i) std::printf("%s%u", i ? ", " : "", h.jgroup_words[i]);
  std::printf("], \"levels\": [");
  for (size_t i = 0; i < h.jgroup_levels.size(); ++i) std::printf("%s%u", i ? ", " : "", h.jgroup_levels[i]);
  std::printf("]}\n");
  return 0;
}
'''


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    d = tmp_path_factory.mktemp("hinge_groups")
    (d / "main.cpp").write_text(HARNESS)
    exe = d / "schedule"
    cuda_inc = "/usr/local/cuda/include"
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{cuda_inc}", f"-I{ROOT / 'include'}", f"-I{CSRC}",
                    str(d / "main.cpp"), str(CSRC / "model.cpp"), str(CSRC / "mjcf.cpp"), "-o", str(exe)],
                   check=True, capture_output=True, timeout=300)
    return d, exe


def scenes():
    from zeno_b200 import scenes as sc
    out = {"ant": sc.ant(), "humanoid": sc.humanoid(), "pendulum": sc.pendulum(), "cartpole": sc.cartpole()}
    for p in sorted((ROOT / "tests" / "golden" / "assets").glob("*.xml")):
        out["asset_" + p.stem] = p.read_text()
    return out


@pytest.mark.parametrize("name", sorted(scenes()))
def test_schedule_reproduces_the_colour_sweep(harness, name):
    d, exe = harness
    xml = d / f"{name}.xml"
    xml.write_text(scenes()[name])
    r = subprocess.run([str(exe), str(xml)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    s = json.loads(r.stdout)
    cons, dyn, groups = s["constraints"], s["dynamic"], s["groups"]
    K = len(cons)
    # (1) every constraint exactly once, in groups of its own pair with the right types
    members = []
    for k0, k1, k2, kind in groups:
        g = [k0] + ([k1] if kind >= 1 else []) + ([k2] if kind == 2 else [])
        if kind >= 1:
            assert [cons[k][2] for k in g] == [2, 3, 4][:len(g)]
            assert len({(cons[k][0], cons[k][1]) for k in g}) == 1
        members.append(g)
    flat = [k for g in members for k in g]
    assert sorted(flat) == list(range(K))
    # (2) per dynamic body, the sweep order (constraint index order) is kept
    for b in range(len(dyn)):
        if not dyn[b]:
            continue
        seq = [k for k in flat if b in cons[k][:2]]
        assert seq == sorted(seq), f"body {b}: {seq}"
    # (3) levels: every group once, disjoint dynamic bodies inside a level, and the
    # level order keeps each dynamic body's group order
    words, levels = np.array(s["words"], np.uint32).reshape(-1, 2), s["levels"]
    if K == 0:
        return
    assert levels[0] == 0 and levels[-1] == len(words) == len(groups)
    by_level = []
    for v in range(len(levels) - 1):
        lv = []
        for w0, w1 in words[levels[v]:levels[v + 1]]:
            lv.append([int(w0 & 0xFFFF), int(w0 >> 16), int(w1 & 0xFFFF), int(w1 >> 16)])
        bodies = [b for g in lv for b in cons[g[0]][:2] if dyn[b]]
        assert len(bodies) == len(set(bodies)), f"level {v} shares a dynamic body"
        by_level.append(lv)
    order = [g for lv in by_level for g in lv]
    assert sorted(map(tuple, order)) == sorted(map(tuple, groups))
    first = {tuple(g): i for i, g in enumerate(groups)}
    for b in range(len(dyn)):
        if not dyn[b]:
            continue
        seq = [first[tuple(g)] for g in order if b in cons[g[0]][:2]]
        assert seq == sorted(seq), f"body {b} out of sweep order across levels"
