"""The caller-side runtime-LoRA config keys, restated from the reference:
the key table (src/ming-model-config-stage.h:33-56), keys forwarded only when
set (src/ming-model-config-stage.cc:177-208), the generator's load-time
reading (src/ming-generator.cc:233-278) and its per-request application
(src/ming-generator.cc:310-337), as the reference's generator test exercises
them (tests/ming-lora-test.cc:268-337: `lora` binds and its strength is live,
a later `lora` path is ignored and said, `lora2` alone takes slot 1)."""
from mingproj import lora_config as LC


def test_key_table_is_positional():
    assert len(LC.CFG_LORA_KEYS) == LC.CFG_LORA_SLOTS == 8
    assert LC.CFG_LORA_KEYS[0] == ("lora", "lora_scale")
    assert LC.CFG_LORA_KEYS[1] == ("lora2", "lora2_scale")
    assert LC.CFG_LORA_KEYS[7] == ("lora8", "lora8_scale")


def test_forwarded_only_when_set():
    assert LC.forwarded_config({}) == {}
    assert LC.forwarded_config(None) == {}
    got = LC.forwarded_config({"lora3": "a.safetensors", "lora3_scale": 0, "lora_scale": -0.5,
                               "shift": 3.0, "lora7": 12})
    # 0 and a negative strength are requests, forwarded as they are; a
    # non-string path is forwarded as the empty string (as_string(""))
    assert got == {"lora3": "a.safetensors", "lora3_scale": 0.0, "lora_scale": -0.5,
                   "lora7": ""}


def test_load_defaults_and_positional_slots():
    files = {"style": "/adapters/style.safetensors"}
    specs, st = LC.load_specs({"lora2": "style", "lora2_scale": 0.5}, files.get)
    assert specs is not None and len(specs) == 8
    assert specs[0].path == "" and specs[0].scale == 1.0     # slot 0 empty, default 1.0
    assert specs[1].path == files["style"] and specs[1].scale == 0.5
    assert all(s.path == "" and s.scale == 1.0 for s in specs[2:])
    assert st.refs[1] == "style" and st.scales == [1.0, 0.5] + [1.0] * 6
    assert st.warnings == []


def test_load_unresolved_and_empty_paths():
    specs, st = LC.load_specs({"lora": "missing", "lora2": "", "lora2_scale": 0.3},
                              lambda ref: None)
    assert specs is None  # nothing resolved: the base model runs
    assert st.scales[1] == 0.3
    assert len(st.warnings) == 1 and "`lora` 'missing' did not resolve" in st.warnings[0]
    assert "NOT applied" in st.warnings[0]


def test_load_slots_past_the_dit_are_said():
    specs, st = LC.load_specs({"lora3": "x", "lora2": "y"}, lambda r: "/f/" + r, slots=2)
    assert specs is not None and len(specs) == 2 and specs[1].path == "/f/y"
    assert any("`lora3` is set, but this host's DiT runs 2 adapters" in w for w in st.warnings)


def test_apply_absent_keys_keep_strengths():
    _, st = LC.load_specs({"lora": "a", "lora_scale": 0.8}, lambda r: "/f/" + r)
    calls = []
    n = LC.apply_keys({"shift": 2.0}, st, lambda i, s: calls.append((i, s)))
    assert n == 0 and calls == [] and st.scales[0] == 0.8


def test_apply_only_changed_strengths_reach_the_dit():
    _, st = LC.load_specs({"lora": "a", "lora_scale": 1.0}, lambda r: "/f/" + r)
    calls = []
    setter = lambda i, s: calls.append((i, s))  # noqa: E731
    assert LC.apply_keys({"lora_scale": 1.0}, st, setter) == 0      # unchanged: no call
    assert LC.apply_keys({"lora_scale": 0.0}, st, setter) == 1      # live strength 0
    assert LC.apply_keys({"lora_scale": 1.0, "lora4_scale": -0.25}, st, setter) == 2
    assert calls == [(0, 0.0), (0, 1.0), (3, -0.25)]
    assert st.scales[0] == 1.0 and st.scales[3] == -0.25


def test_apply_path_change_is_ignored_and_said_once():
    _, st = LC.load_specs({"lora": "a"}, lambda r: "/f/" + r)
    calls = []
    beat = {"lora": "/nonexistent/x.safetensors", "lora_scale": 0.5}
    LC.apply_keys(beat, st, lambda i, s: calls.append((i, s)), modules=lambda i: 238)
    LC.apply_keys(beat, st, lambda i, s: calls.append((i, s)))
    assert st.refs[0] == "a"                       # the loaded adapter stays
    assert len(st.warnings) == 1 and "is IGNORED" in st.warnings[0]
    assert "`lora_scale` still applies" in st.warnings[0]
    assert calls == [(0, 0.5)]                     # the strength still applies
    assert st.infos == ["ming-image: `lora_scale` -> 0.500 (238 modules)"]
    # naming the loaded adapter again says nothing
    LC.apply_keys({"lora": "a"}, st, lambda i, s: None)
    assert len(st.warnings) == 1
