"""The C ABI from C (no GPU needed): tests/c_abi_smoke.c is compiled with gcc against
include/hive_b200.h and linked to libhive_b200.so, so the header's declarations, the
exported symbols and the status/last-error convention are checked the way a C or cgo
caller meets them."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def smoke_bin(tmp_path_factory):
    import build
    lib = build.build()
    if shutil.which("gcc") is None:
        pytest.skip("gcc not found")
    out = tmp_path_factory.mktemp("cabi") / "c_abi_smoke"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", f"-I{REPO / 'include'}",
                    str(REPO / "tests" / "c_abi_smoke.c"), "-o", str(out),
                    f"-L{lib.parent}", "-lhive_b200", f"-Wl,-rpath,{lib.parent}"],
                   check=True)
    return out


def test_c_caller_sees_the_abi(smoke_bin):
    r = subprocess.run([str(smoke_bin)], capture_output=True, text=True, timeout=120,
                       env=dict(os.environ))
    assert r.returncode == 0, r.stderr
    kv = dict(line.split("=", 1) for line in r.stdout.splitlines() if "=" in line)
    assert kv["version"] == kv["abi_macro"]
    assert kv["has_k_step"] == "1"
    assert kv["a4gv_null_rc"] == "1001" and "bad arguments" in kv["a4gv_null_msg"]
    assert kv["wait_probe_null_rc"] == "1001"
    assert kv["argmax_key_final_null_rc"] == "1001"
    assert kv["prepacked_rc"].startswith("0 ")
    assert kv["init_msg_nonempty"] == "1"
