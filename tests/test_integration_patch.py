"""CPU checks of integration/nx_vulkan_b200.patch, the edits that route the
reference's Elixir host layer to the new nxv_* entry points (reviewed here,
not executed: there is no Elixir or Rust toolchain in this image).

  * every `extern "C"` declaration the patch adds to lib.rs names a symbol
    of include/nx_vulkan_shim.h with the same number of parameters;
  * every NIF the patch adds has a stub in native.ex with the same arity
    (the NIF's parameters minus `env`), and the Elixir wrappers call stubs
    that exist, with that arity;
  * the compiler routes scalar literals to immediates and every 4-input
    chain to fused_chain_imm; the backend routes argmax, f64 reductions and
    f64 / batched dot to the new wrappers;
  * the patch applies cleanly to the reference sources when they are present.
"""
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from conftest import ROOT

PATCH = (ROOT / "integration" / "nx_vulkan_b200.patch").read_text()
HEADER = (ROOT / "include" / "nx_vulkan_shim.h").read_text()
REFERENCE = Path("/root/reference")


def added(path):
    """The lines the patch adds to `path` (without the leading '+')."""
    out, cur = [], None
    for line in PATCH.splitlines():
        if line.startswith("+++ "):
            cur = line[4:].split("\t")[0]
            continue
        if cur and cur.endswith(path) and line.startswith("+") and not line.startswith("+++"):
            out.append(line[1:])
    return "\n".join(out)


def c_params(decl_args: str) -> int:
    decl_args = decl_args.strip()
    return 0 if decl_args in ("", "void") else decl_args.count(",") + 1


def header_arity():
    body = re.sub(r"/\*.*?\*/", "", HEADER, flags=re.S)
    return {m.group(1): c_params(m.group(2))
            for m in re.finditer(r"\b(nxv_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", body, flags=re.S)}


def test_extern_declarations_match_the_header():
    rs = added("src/lib.rs")
    decls = re.findall(r"fn (nxv_[a-z0-9_]+)\(([^;]*?)\)\s*->", rs, flags=re.S)
    assert len(decls) >= 10
    hdr = header_arity()
    for name, args in decls:
        assert name in hdr, name
        n = len([a for a in args.split(",") if a.strip()])
        assert n == hdr[name], (name, n, hdr[name])


def nif_arity():
    rs = added("src/lib.rs")
    out = {}
    for m in re.finditer(r"#\[rustler::nif[^\]]*\]\s*fn ([a-z0-9_]+)<'a>\((.*?)\)\s*->", rs, flags=re.S):
        params = [p for p in m.group(2).split(",") if p.strip()]
        assert params[0].strip().startswith("env")
        out[m.group(1)] = len(params) - 1
    return out


def test_every_nif_has_a_stub_of_the_same_arity():
    stubs = {m.group(1): c_params(m.group(2))
             for m in re.finditer(r"def ([a-z0-9_]+)\(([^)]*)\)", added("native.ex"))}
    nifs = nif_arity()
    assert len(nifs) >= 10
    for name, n in nifs.items():
        assert stubs.get(name) == n, (name, n, stubs.get(name))


def test_wrappers_call_existing_stubs():
    stubs = {m.group(1): c_params(m.group(2))
             for m in re.finditer(r"def ([a-z0-9_]+)\(([^)]*)\)", added("native.ex"))}
    ex = added("lib/nx_vulkan.ex")
    calls = re.findall(r"Nx\.Vulkan\.Native\.([a-z0-9_]+)\(", ex)
    assert set(calls) <= set(stubs), set(calls) - set(stubs)
    for name in ("fused_chain_imm", "argmax_axis", "matmul_batched", "reduce_f64",
                 "leapfrog_chain_gauss_f64_batched", "leapfrog_logreg_f64_batched"):
        assert name in calls, name


def test_routing_edits():
    comp = added("compiler.ex")
    assert "op: :constant" in comp and "{:imm, v * 1.0}" in comp
    assert "Nx.Vulkan.fused_chain_imm(ar, [br, cr, dr], ops_with_buf, out_type)" in comp
    be = added("backend.ex")
    assert "Nx.Vulkan.argmax_axis(" in be
    assert "Nx.Vulkan.reduce_f64(" in be
    assert "Nx.Vulkan.matmul_batched(" in be
    assert "NXV_B200_LIB_DIR" in added("build.rs")


@pytest.mark.skipif(not REFERENCE.exists() or shutil.which("patch") is None,
                    reason="reference sources or patch(1) not present")
def test_patch_applies_to_the_reference(tmp_path):
    for line in PATCH.splitlines():
        if line.startswith("--- a/"):
            rel = line[6:].split("\t")[0]
            (tmp_path / rel).parent.mkdir(parents=True, exist_ok=True)
            shutil.copy(REFERENCE / rel, tmp_path / rel)
    r = subprocess.run(["patch", "-p1", "--dry-run", "-i", str(ROOT / "integration" / "nx_vulkan_b200.patch")],
                       cwd=tmp_path, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
