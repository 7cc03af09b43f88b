"""The C ABI library without a GPU: it loads, exports every function that
include/zs_sampler.h declares, the zen:: C++ API of include/zen/sample.h links
and runs its host-only parts, and argument errors come back as statuses."""

import ctypes as C
import os
import re
import subprocess

import pytest

from zeninfer_b200 import Rng, SamplingParams, _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "zs_sampler.h")


@pytest.fixture(scope="module")
def lib():
    from zeninfer_b200 import build
    build.build_sampler()
    return _native.lib()


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"^(?:zs_status|const char\s*\*|int|uint64_t)\s+(zs_\w+)\s*\(", text,
                          re.M))


def test_header_declares_the_bound_set():
    names = _declared()
    assert "zs_sample" in names and "zs_sample_noalloc" in names
    assert names == set(_native.EXPORTS)


def test_every_declared_symbol_is_exported(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _native.SAMPLER_SO], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (\w+)$", out, re.M))
    missing = _declared() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_version_and_strings(lib):
    ver = int(re.search(r"#define ZS_ABI_VERSION (\d+)", open(HEADER).read()).group(1))
    assert lib.zs_abi_version() == ver
    for s in range(7):
        assert lib.zs_status_string(s)
    assert lib.zs_status_string(0) == b"ok"


def test_rng_seed(lib):
    assert lib.zs_rng_seed(0) == 0x9E3779B97F4A7C15
    for s in (1, 42, (1 << 64) - 1):
        assert lib.zs_rng_seed(s) == s == Rng(s).state


def test_argument_errors_need_no_device(lib):
    p = SamplingParams(temp=0.7, top_k=40).to_c()
    # null handle
    assert lib.zs_sample(None, None, 0, 1, 1, C.byref(p), 0, None, 0, None, None, None, None,
                         None) == 1
    assert "null handle" in lib.zs_last_error().decode()
    # batch 0 is a no-op; null params is an error
    assert lib.zs_sample_noalloc(None, 0, 0, 10, C.byref(p), None, 0, None, None, None, None,
                                 None) == 0
    assert lib.zs_sample_noalloc(None, 0, 1, 10, None, None, 0, None, None, None, None,
                                 None) == 1
    out = C.c_int64()
    assert lib.zs_shard_partial_bytes(4, 0, 2, C.byref(p), 0, C.byref(out)) == 1
    assert lib.zs_set_lmhead_route(None, 0) == 1
    assert lib.zs_set_lmhead_tiles(None, 0) == 1


def test_create_without_device(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    h = C.c_void_p()
    assert lib.zs_create(0, C.byref(h)) == 3  # ZS_ERR_NO_DEVICE
    assert not h.value


def test_shard_layout_is_rank_independent(lib):
    """Every rank derives the same block size from (batch, V, G, params) alone."""
    p = SamplingParams(temp=0.7, top_k=50, top_p=0.9).to_c()
    sizes = []
    for batch in (1, 7, 256, 4096):
        out = C.c_int64()
        assert lib.zs_shard_partial_bytes(batch, 151936, 8, C.byref(p), 0, C.byref(out)) == 0
        assert out.value > 0 and out.value % 16 == 0
        sizes.append(out.value)
    assert sizes[-1] >= sizes[-2]


CPP_PROGRAM = r"""
#include <cstdio>
#include <stdexcept>
#include <vector>
#include "zen/sample.h"
int main() {
    zen::Rng rng(42);
    for (int i = 0; i < 3; ++i) std::printf("%llu\n", (unsigned long long)rng.next());
    zen::Rng z(0);
    std::printf("%.17g\n", z.uniform());
    // the reference's call pattern (src/main.cpp:615-628)
    zen::SamplingParams sp;
    sp.temp = 0.7f;
    sp.top_k = 40;
    std::vector<int32_t> history;
    std::vector<float> logits(1000, 0.0f);
    logits[17] = 5.0f;
    try {
        int id = zen::sample_token(logits.data(), (int)logits.size(), sp, history, rng);
        std::printf("id %d\n", id);
    } catch (const std::exception& e) {
        std::printf("error: %s\n", e.what());
    }
    return 0;
}
"""


def test_cpp_api_links_and_runs(lib, tmp_path):
    src = tmp_path / "use_sample.cpp"
    src.write_text(CPP_PROGRAM)
    exe = tmp_path / "use_sample"
    libdir = os.path.dirname(_native.SAMPLER_SO)
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{ROOT}/include", str(src), "-o", str(exe),
                    f"-L{libdir}", "-lzs_sampler", f"-Wl,-rpath,{libdir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    r = Rng(42)
    assert [int(v) for v in out[:3]] == [r.next() for _ in range(3)]
    assert float(out[3]) == Rng(0).uniform()
    assert out[4].startswith("id ") or out[4].startswith("error: ")
