"""CPU checks of the C ABI: the library loads, exports every entry point that
include/b200_sampler.h declares, and its structs match the reference layout."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "b200_sampler.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(bs_[a-z_0-9]+)\s*\(", src)))


def test_library_builds_and_exports_every_declared_symbol(pkg):
    pkg.build.build()
    L = pkg.lib()
    names = declared_functions()
    assert "bs_create" in names and "bs_sample" in names
    for n in names:
        assert hasattr(L, n), f"missing export {n}"
    assert set(pkg.EXPORTS) <= set(names)


def test_config_layout_matches_samplerconfig(pkg, orc):
    from_lib = pkg.sampler.BsConfig
    assert ctypes.sizeof(from_lib) == 40
    assert ctypes.sizeof(orc.OrcConfig) == 40
    for (a, ta), (b, tb) in zip(from_lib._fields_, orc.OrcConfig._fields_):
        assert a == b and ta == tb
        assert getattr(from_lib, a).offset == getattr(orc.OrcConfig, b).offset
    assert from_lib.seed.offset == 24


def test_config_defaults_match_reference(pkg):
    c = pkg.sampler.BsConfig()
    pkg.lib().bs_config_default(ctypes.byref(c))
    ref = pkg.SamplerConfig()   # sampler.zig:5-12
    assert abs(c.temperature - ref.temperature) < 1e-7 and c.top_k == ref.top_k
    assert abs(c.top_p - ref.top_p) < 1e-7 and c.min_p == ref.min_p and c.typical_p == ref.typical_p
    assert c.seed == 0 and c.repetition_window == 32 and abs(c.repetition_penalty - 1.1) < 1e-7


def test_status_strings(pkg):
    assert pkg.status_string(0) == "ok"
    assert "memory" in pkg.status_string(2)


def test_invalid_arguments_are_rejected_without_gpu(pkg):
    L = pkg.lib()
    c = pkg.SamplerConfig().to_c()
    h = ctypes.c_void_p()
    assert L.bs_create(ctypes.byref(c), 0, 100, 0, None, ctypes.byref(h)) == 1   # batch 0
    assert L.bs_create(None, 1, 100, 0, None, ctypes.byref(h)) == 1
    assert L.bs_sample(None, None, 0, 0, 1, None, 0, None, None) == 1
    assert L.bs_argmax(None, 0, 1, 10, None, None) == 1


# SplitMix64 (Steele, Lea & Flood) from x = 1234567: the published first
# outputs of the reference implementation.  Sampler.init's DefaultPrng takes
# its four state words from these (sampler.zig:22).
SPLITMIX64_1234567 = [6457827717110365317, 3203168211198807973, 9817491932198370423,
                      4593380528125082431, 16408922859458223821]


def test_seed_state_is_splitmix64_on_the_host(pkg, orc):
    st = pkg.sampler.seed_state(1234567)
    assert [int(v) for v in st] == SPLITMIX64_1234567[:4]
    assert [int(v) for v in orc.rng_seed(1234567)] == SPLITMIX64_1234567[:4]
    # seed 0 is replaced by 0xDEADBEEF (sampler.zig:22)
    assert list(pkg.sampler.seed_state(0)) == list(pkg.sampler.seed_state(0xDEADBEEF))
    for seed in (1, 42, 2**63 + 5, 2**64 - 1):
        assert list(pkg.sampler.seed_state(seed)) == list(orc.rng_seed(seed))
    assert pkg.lib().bs_seed_state(0, None) == 1


def test_sampler_init_needs_no_device(pkg):
    # Sampler.init(cfg) (sampler.zig:19-24) takes no vocabulary and does no
    # device work: the handle is made by the first sample
    s = pkg.Sampler.init(pkg.SamplerConfig(seed=1234567))
    assert not s._h and s.vocab == 0
    assert [int(v) for v in s.rng_state[0]] == SPLITMIX64_1234567[:4]
    s.rng_state = [[1, 2, 3, 4]]
    assert [int(v) for v in s.rng_state[0]] == [1, 2, 3, 4]
