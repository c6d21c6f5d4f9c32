"""The drop-in boundary without a GPU: the library loads, exports every entry point include/ntc_b200.h
declares and every ntc_cuda::Trainer member the reference trainer calls, and the description structs
have the reference header's layout (main.cpp fills them by field name)."""
import ctypes as C
import os
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from neural_block_textures_b200 import abi

ROOT = Path(__file__).resolve().parent.parent
# The reference tree (read-only, present where the oracle is built; NTC_REFERENCE names it, as __graft_entry__ reads it).
REF_HEADER = Path(os.environ.get("NTC_REFERENCE", "/root/reference")) / "cuda" / "ntc_cuda.h"
LIB = abi.LIB_PATH


def header_functions() -> list[str]:
    text = (ROOT / "include" / "ntc_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ntcb_\w+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = abi.load_library()
    names = header_functions()
    assert len(names) >= 30
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ntc_b200.h but not exported"
    assert set(names) == set(abi.SIGNATURES), "abi.py binds exactly the header's entry points"


def _defined_dynamic_symbols(path: Path) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True, check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if ln.strip()}


def test_cxx_trainer_symbols_cover_the_reference_callers():
    """Every ntc_cuda:: symbol the reference main.cpp (compiled with NTC_CUDA=1) needs is defined by libntc_b200.so."""
    obj = ROOT / "oracle" / "_ref" / "main_cuda.o"
    if not obj.exists():
        pytest.skip("oracle/_ref/main_cuda.o not built (needs the reference tree)")
    und = subprocess.run(["nm", "-u", str(obj)], capture_output=True, text=True, check=True).stdout
    need = {ln.split()[-1] for ln in und.splitlines() if "ntc_cuda" in ln}
    assert len(need) >= 20
    have = _defined_dynamic_symbols(LIB)
    missing = need - have
    assert not missing, f"unresolved Trainer members: {sorted(missing)}"


LAYOUT_PROBE = r"""
#include <cstddef>
#include <cstdio>
#include HEADER
#define F(S, f) std::printf("%s.%s %zu\n", #S, #f, offsetof(ntc_cuda::S, f));
int main() {
  std::printf("sizeof.LevelDesc %zu\nsizeof.ModelDesc %zu\nsizeof.QesDesc %zu\nsizeof.DctDesc %zu\n",
              sizeof(ntc_cuda::LevelDesc), sizeof(ntc_cuda::ModelDesc), sizeof(ntc_cuda::QesDesc), sizeof(ntc_cuda::DctDesc));
  F(LevelDesc, W) F(LevelDesc, off) F(LevelDesc, nearest)
  F(ModelDesc, W) F(ModelDesc, T) F(ModelDesc, nlev) F(ModelDesc, lv) F(ModelDesc, npos) F(ModelDesc, pos) F(ModelDesc, nin)
  F(ModelDesc, nout) F(ModelDesc, nhidden) F(ModelDesc, hidden) F(ModelDesc, leak) F(ModelDesc, clamp_out) F(ModelDesc, cw)
  F(ModelDesc, wsum) F(ModelDesc, qat_bits) F(ModelDesc, qat) F(ModelDesc, qat_grid) F(ModelDesc, qes_bits) F(ModelDesc, dct)
  F(ModelDesc, dct_C) F(ModelDesc, dct_N) F(ModelDesc, dct_dc_step) F(ModelDesc, dct_q) F(ModelDesc, dct_basis)
  F(ModelDesc, dct_zigzag) F(ModelDesc, max_pairs) F(ModelDesc, max_batch) F(ModelDesc, seed)
  F(QesDesc, bits) F(QesDesc, live) F(QesDesc, frozen) F(QesDesc, lo) F(QesDesc, hi) F(QesDesc, range) F(QesDesc, grid_off)
  F(DctDesc, live) F(DctDesc, rate_es) F(DctDesc, rate_scale) F(DctDesc, lam_t16) F(DctDesc, lo_w16) F(DctDesc, deadzone)
  return 0;
}
"""


def _layout(header: Path, tmp_path: Path) -> dict[str, int]:
    if not shutil.which("g++"):
        pytest.skip("no g++")
    src = tmp_path / "probe.cpp"
    src.write_text(LAYOUT_PROBE.replace("HEADER", f'"{header}"'))
    exe = tmp_path / f"probe_{header.parent.name}"
    subprocess.run(["g++", "-std=c++17", "-o", str(exe), str(src)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    return {k: int(v) for k, v in (ln.split() for ln in out.splitlines())}


def test_struct_layout_matches_reference_header(tmp_path):
    ours = _layout(ROOT / "include" / "ntc_cuda.h", tmp_path)
    if not REF_HEADER.exists():
        pytest.skip("reference tree absent")
    (tmp_path / "ref").mkdir()
    theirs = _layout(REF_HEADER, tmp_path / "ref")
    assert ours == theirs


def test_ctypes_layout_matches_c_header(tmp_path):
    ours = _layout(ROOT / "include" / "ntc_cuda.h", tmp_path)
    assert C.sizeof(abi.ModelDesc) == ours["sizeof.ModelDesc"]
    assert C.sizeof(abi.LevelDesc) == ours["sizeof.LevelDesc"]
    assert C.sizeof(abi.QesDesc) == ours["sizeof.QesDesc"]
    assert C.sizeof(abi.DctDesc) == ours["sizeof.DctDesc"]
    for key, off in ours.items():
        s, f = key.split(".")
        if s == "sizeof":
            continue
        cls = {"LevelDesc": abi.LevelDesc, "ModelDesc": abi.ModelDesc, "QesDesc": abi.QesDesc, "DctDesc": abi.DctDesc}[s]
        assert getattr(cls, f).offset == off, key


def test_progress_stats_layout_matches_c_header(tmp_path):
    """ctypes ProgressStats against ntcb_progress_stats as the C compiler lays it out."""
    if not shutil.which("gcc"):
        pytest.skip("no gcc")
    fields = [f for f, _ in abi.ProgressStats._fields_]
    src = tmp_path / "ps.c"
    src.write_text("#include <stddef.h>\n#include <stdio.h>\n#include \"%s\"\nint main(void) {\n"
                   "  printf(\"sizeof %%zu\\n\", sizeof(ntcb_progress_stats));\n%s  return 0;\n}\n"
                   % (ROOT / "include" / "ntc_b200.h",
                      "".join('  printf("%s %%zu\\n", offsetof(ntcb_progress_stats, %s));\n' % (f, f) for f in fields)))
    exe = tmp_path / "ps"
    subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True)
    out = dict(ln.split() for ln in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines())
    assert int(out["sizeof"]) == C.sizeof(abi.ProgressStats)
    for f in fields:
        assert getattr(abi.ProgressStats, f).offset == int(out[f]), f


def test_init_without_gpu_reports_a_reason(tmp_path):
    """On a machine without a CUDA device init() returns false with a reason instead of crashing (run in a child)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("this machine has a GPU")
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "from neural_block_textures_b200 import Trainer\n"
        "from tests.helpers import spec_named, target_for\n"
        "s = spec_named('cfg1'); z, p = s.init_params(); t = Trainer()\n"
        "ok, why = t.init(s.model_desc(), z, p, target_for(s)); print(ok, why)\n" % str(ROOT))
    r = subprocess.run(["python", "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.startswith("False") and "CUDA" in r.stdout
