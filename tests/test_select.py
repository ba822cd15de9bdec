"""Variant spaces and selections in the C++ host library, against the
reference's own golden texts (test/Test/FuryKernel/JsonTest.hs,
VariantTest.hs, SelectionTest.hs) where they do not depend on the eDSL's
kernels, and this target's GEMV family (one axis, the split-K) where they
do."""

import json
import random

import pytest

from furykernel_b200 import _host as H
from furykernel_b200 import _native as N
from tests.restated import lowering as RL

# ---------------------------------------------------------------------------
# JSON (JsonTest.hs)


def render(v, depth=0) -> str:
    """The reference's layout (Json.hs renderJson), restated for the test."""
    pad, close = "  " * (depth + 1), "  " * depth

    def s(t):
        out = '"'
        for c in t:
            out += {'"': '\\"', "\\": "\\\\", "\n": "\\n", "\r": "\\r", "\t": "\\t"}.get(
                c, "\\u%04x" % ord(c) if ord(c) < 0x20 else c)
        return out + '"'

    if v is None:
        return "null"
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, int):
        return str(v)
    if isinstance(v, str):
        return s(v)
    if isinstance(v, list):
        return "[]" if not v else "[\n" + ",\n".join(pad + render(x, depth + 1) for x in v) + "\n" + close + "]"
    return "{}" if not v else "{\n" + ",\n".join(pad + s(k) + ": " + render(x, depth + 1)
                                                 for k, x in v.items()) + "\n" + close + "}"


def random_json(rng, depth=0):
    kind = rng.randrange(6 if depth < 3 else 4)
    if kind == 0:
        return None
    if kind == 1:
        return rng.random() < 0.5
    if kind == 2:
        return rng.randrange(-(2 ** 63), 2 ** 63)
    if kind == 3:
        return "".join(rng.choice('ab"\\/\n\t\r\b\f\x00é😀') for _ in range(rng.randrange(9)))
    if kind == 4:
        return [random_json(rng, depth + 1) for _ in range(rng.randrange(6))]
    return {"".join(rng.choice("abc\"\n") for _ in range(rng.randrange(1, 5))): random_json(rng, depth + 1)
            for _ in range(rng.randrange(6))}


def test_what_is_written_reads_back():
    rng = random.Random(8259)
    for _ in range(300):
        text = render(random_json(rng)) + "\n"
        assert H.json_roundtrip(text) == text


def test_escapes_surrogate_pairs_whitespace():
    got = H.json_roundtrip(' { "a\\"b\\\\c\\/d\\u00e9\\ud83d\\ude00" : [ -12 , true , null ] } ')
    assert json.loads(got) == {'a"b\\c/dé\U0001F600': [-12, True, None]}
    assert H.json_roundtrip("[]") == "[]\n" and H.json_roundtrip("{}") == "{}\n"


@pytest.mark.parametrize("text,error", [
    ('{"a": 1, "a": 2}', "The key a twice at character 9."),
    ("1.5", "A number that is not an integer at character 1."),
    ("[1 2]", "No , or ] after an element at character 3."),
    ("01", "A leading zero at character 0."),
    ('"\\ud800"', "A lone surrogate at character 7."),
    ('"a\nb"', "A control character in a string at character 2."),
    ("true false", "Text after the value at character 5."),
    ("", "No JSON value at character 0."),
])
def test_what_is_not_json_and_where(text, error):
    with pytest.raises(N.Refused) as e:
        H.json_roundtrip(text)
    assert str(e.value).endswith(error)


# ---------------------------------------------------------------------------
# Variant spaces (VariantTest.hs): axis keys, names, checkSpace

GEMV_AXES = [{"name": "rows_per_simd", "prefix": "r", "values": [1, 2, 4, 8], "order": False},
             {"name": "threads", "prefix": "t", "values": [32, 64, 128, 256, 512, 1024], "order": False},
             {"name": "pack", "prefix": "p", "values": [4, 8, 16], "order": True},
             {"name": "split_k", "prefix": "s", "values": [1, 2, 4, 8, 16], "order": True}]


def space(family="gemv", axes=None, classes=None, batch=("m",)):
    return json.dumps({"family": family, "axes": GEMV_AXES if axes is None else axes,
                       "classes": classes if classes is not None else [{"n": 8, "k": 256, "m": 1}],
                       "batch": list(batch)})


def err(f, *a):
    with pytest.raises(N.Refused) as e:
        f(*a)
    return str(e.value)


def test_axis_keys_read_back_and_say_what_is_wrong():
    assert H.space_parse_key(space(), "r2_t128_p8_s1") == "r2_t128_p8_s1"
    assert err(H.space_parse_key, space(), "r2_t128") == "The axis key r2_t128 has 2 parts for 4 axes."
    assert err(H.space_parse_key, space(), "r2_x128_p8_s1") == \
        "The axis key r2_x128_p8_s1 has x128 where threads (t) belongs."
    assert err(H.space_parse_key, space(), "r3_t128_p8_s1") == \
        "The axis key r3_t128_p8_s1 gives rows_per_simd 3, which is not one of its values."
    assert err(H.space_parse_key, space(), "r01_t128_p8_s1") == \
        "The axis key r01_t128_p8_s1 writes rows_per_simd 1 as 01."
    assert H.space_parse_key(space(axes=[]), "") == ""


def test_names_and_that_they_read_back():
    names = H.space_names(space(classes=[{"n": 8, "k": 256, "m": 1}, {"n": 8, "k": 256, "m": 2},
                                         {"n": 16, "k": 512, "m": 1}]))
    assert len(names) == 3 * 4 * 6 * 3 * 5
    assert "gemv_n8_k256_m1_x_r1_t32_p8_s1" in names
    assert not [n for n in names if "does not read back" in n]
    assert H.space_names(space(axes=[])) == ["gemv_n8_k256_m1"]
    assert H.space_names(space(classes=[{}])) [0] == "gemv_x_r1_t32_p4_s1"


def test_names_split_back_at_the_first_x_whose_right_side_is_valid():
    assert H.split_join("model_embed_x_s0_x_x_m1", "m") == ("model_embed_x_s0_x", "m1")
    assert H.split_join("a_x_b_x_m16", "m") == ("a_x_b", "m16")
    assert H.split_join("a_x_b", "m") is None


def test_spaces_whose_names_would_not_read_back():
    assert H.space_check(space()) == []
    assert H.space_check(space(family="gemv_x_wide")) == \
        ["The family gemv_x_wide holds _x_, which joins a variant's name to its axis key."]
    assert H.space_check(space(axes=GEMV_AXES + [{"name": "unused", "prefix": "r", "values": [1], "order": False}])) \
        == ["The axes rows_per_simd and unused share the prefix r."]
    assert H.space_check(space(axes=[{"name": "rows", "prefix": "r_", "values": [1], "order": False},
                                     {"name": "none", "prefix": "n", "values": [], "order": False}])) == \
        ['The axis rows\'s prefix "r_" is not lowercase letters.', "The axis none has no values."]
    assert H.space_check(space(batch=["mm"])) == \
        ["The batch dimension mm is not a dimension of the class n8_k256_m1."]


def test_classes_that_would_be_misread():
    # VariantTest.hs: a class as pairs, so that it can give a dimension twice.
    classes = [[["n", 8], ["k_", 256], ["m", 1]], [["n", 8], ["n", 16], ["m", 1]], {"n": 8, "k": 256, "m": 1},
               {"n": 8, "k": 256, "m": 1}]
    assert H.space_check(space(classes=classes, batch=())) == [
        'The class n8_k_256_m1\'s dimension "k_" is not lowercase letters.',
        "The class n8_n16_m1 gives n 2 times.",
        "The class n8_k256_m1 is given 2 times."]


# ---------------------------------------------------------------------------
# Selections (SelectionTest.hs): the format, golden

GOLDEN = "\n".join([
    "{",
    '  "format": "furykernel-selection",',
    '  "version": 1,',
    '  "family": "gemv",',
    '  "target": "T32",',
    '  "profile": {',
    '    "cores": 2',
    "  },",
    '  "classes": {',
    '    "n8_k256_m1": {',
    '      "variant": "r1_t32_p8_s1",',
    '      "ir_hash": "0xfedcba9876543210"',
    "    },",
    '    "n8_k256_m2": {',
    '      "variant": "r1_t64_p8_s1",',
    '      "ir_hash": "0x0123456789abcdef"',
    "    }",
    "  }",
    "}",
]) + "\n"


def test_the_format_classes_in_key_order():
    # Written in the other order, it renders in key order.
    shuffled = GOLDEN.replace('"n8_k256_m1"', '"TMP"').replace('"n8_k256_m2"', '"n8_k256_m1"')
    shuffled = shuffled.replace('"TMP"', '"n8_k256_m2"')
    shuffled = shuffled.replace("0xfedcba9876543210", "X").replace("0x0123456789abcdef", "0xfedcba9876543210")
    shuffled = shuffled.replace("X", "0x0123456789abcdef").replace('"r1_t32_p8_s1"', '"Y"')
    shuffled = shuffled.replace('"r1_t64_p8_s1"', '"r1_t32_p8_s1"').replace('"Y"', '"r1_t64_p8_s1"')
    assert H.selection_roundtrip(shuffled) == GOLDEN
    assert H.selection_roundtrip(GOLDEN) == GOLDEN


def field(name, value):
    fields = [("format", '"furykernel-selection"'), ("version", "1"), ("family", '"gemv"'), ("target", '"T32"'),
              ("profile", '{"cores": 2}'), ("classes", "{}")]
    return "{" + ", ".join(f'"{k}": {value if k == name else v}' for k, v in fields) + "}"


@pytest.mark.parametrize("text,error", [
    ("[]", "A selection is a JSON object."),
    (field("format", '"other"'), "The format is other, not furykernel-selection."),
    (field("version", "2"), "Version 2 of the format; this reads version 1."),
    ('{"format": "furykernel-selection", "version": 2, "extra": 1}', "Version 2 of the format; this reads version 1."),
    (field("classes", '{"n8_k256_m1": "r1_t32_p8_s1"}'), "The field classes has the wrong type."),
    (field("classes", '{"n8_k256_m1": {"variant": "r1_t32_p8_s1", "ir_hash": "0x12"}}'),
     "The field classes has the wrong type."),
    (field("profile", '{"cores": -1}'), "The field profile has the wrong type."),
    ('{"format": "furykernel-selection", "version": 1, "extra": 1}', "An unknown field: extra."),
    ('{"format": "furykernel-selection", "version": 1}', "The field family is missing."),
])
def test_the_format_is_checked(text, error):
    assert err(H.selection_roundtrip, text) == error


# ---------------------------------------------------------------------------
# This target's GEMV family: one axis, the split-K, which orders the reduction

CORES = 148
LLAMA = [(12288, 4096), (4096, 4096), (22016, 4096), (4096, 11008), (32000, 4096)]


def test_the_kernel_a_point_runs_and_its_parallelism():
    assert H.gemv_consider(11008, 4096, 1, 1, CORES)[:2] == ("kept", 11008)   # streaming: rows
    assert H.gemv_consider(11008, 4096, 16, 1, CORES)[:2] == ("kept", 2752)   # batched: 4-row groups
    assert H.gemv_consider(11008, 4096, 16, 2, CORES)[:2] == ("kept", 2752)   # chunked: 8 / s rows a block
    assert H.gemv_consider(512, 512, 16, 1, CORES)[:2] == ("too few", 128)
    assert H.gemv_consider(512, 512, 16, 8, CORES)[:2] == ("kept", 512)
    assert H.gemv_consider(100, 1002, 1, 1, CORES)[0] == "indivisible"
    assert H.gemv_consider(100, 1000, 65, 1, CORES)[0] == "illegal"
    # The streaming kernel at split 2 and the batched at split 1 are other kernels.
    hashes = {H.gemv_consider(4096, 4096, m, s, CORES)[2] for m in (1, 16) for s in (1, 2)}
    assert len(hashes) == 4


def llama_classes(batches):
    return [(n, k, m) for n, k in LLAMA for m in batches]


def test_a_selection_reads_back_and_gives_each_class_its_split():
    classes = llama_classes((1, 4, 16, 32))
    text = H.gemv_selection_render(classes, [1] * len(classes), CORES)
    assert text.startswith('{\n  "format": "furykernel-selection",\n  "version": 1,\n  "family": "gemv",\n'
                           '  "target": "Cuda",\n  "profile": {\n    "cores": 148\n  },')
    assert H.selection_roundtrip(text) == text
    assert H.gemv_selection_validate(text, classes, CORES) == [1] * len(classes)


def test_the_batch_sizes_of_a_class_share_the_order_of_its_reductions():
    classes = [(4096, 11008, 1), (4096, 11008, 16)]
    with pytest.raises(N.Refused):  # rendering validates: two splits for one (n, k)
        H.gemv_selection_render(classes, [1, 2], CORES)
    # A selection written with them is refused with the reference's words.
    a = H.gemv_selection_render(classes[:1], [1], CORES)
    b = H.gemv_selection_render(classes[1:], [2], CORES)
    merged = json.loads(a)
    merged["classes"].update(json.loads(b)["classes"])
    assert err(H.gemv_selection_validate, json.dumps(merged), classes, CORES) == (
        "The classes n4096_k11008_m1 and n4096_k11008_m16 differ only in batch size, and order reductions "
        "differently: s1 against s2.")


def test_everything_else_validation_refuses():
    classes = llama_classes((1,))
    good = json.loads(H.gemv_selection_render(classes, [1] * len(classes), CORES))
    wrong = dict(good, family="gemm", target="T64", classes={})
    assert err(H.gemv_selection_validate, json.dumps(wrong), classes, CORES).split("\n") == [
        "The selection is for the family gemm, not gemv.",
        "The selection is for the target T64, not Cuda."] + [
        f"No variant for the class n{n}_k{k}_m1." for n, k, _ in classes]
    assert err(H.gemv_selection_validate, json.dumps(good), classes, 132) == \
        "The selection was made for a GPU of 148 cores, not 132."
    stale = json.loads(json.dumps(good))
    stale["classes"]["n4096_k4096_m1"]["ir_hash"] = "0x0000000000000001"
    msg = err(H.gemv_selection_validate, json.dumps(stale), classes, CORES)
    assert msg.startswith("gemv_n4096_k4096_m1_x_s1 was picked as the kernel of IR hash 0x0000000000000001, "
                          "and is now 0x")
    odd = json.loads(json.dumps(good))
    odd["classes"]["n4096_k4096_m1"]["variant"] = "s3"
    odd["classes"]["n9_k256_m1"] = {"variant": "s1", "ir_hash": "0x0000000000000000"}
    assert err(H.gemv_selection_validate, json.dumps(odd), classes, CORES).split("\n") == [
        "The class n9_k256_m1 is not one of the family's.",
        "The class n4096_k4096_m1's axis key s3 gives split_k 3, which is not one of its values."]
    small = [(512, 512, 16)]
    few = {"format": "furykernel-selection", "version": 1, "family": "gemv", "target": "Cuda",
           "profile": {"cores": CORES}, "classes": {"n512_k512_m16": {"variant": "s1", "ir_hash": "0x" + "0" * 16}}}
    assert err(H.gemv_selection_validate, json.dumps(few), small, CORES) == \
        "gemv_n512_k512_m16_x_s1 launches 128 threadgroups, fewer than twice the 148 cores."


# ---------------------------------------------------------------------------
# The engine under a selection (launch lists only; nothing runs)


def test_the_engine_takes_each_shape_s_split_from_a_selection():
    from furykernel_b200 import select
    from furykernel_b200.shape import LlamaShape
    from tests.test_host_cpp import fake_engine

    s = LlamaShape(layers=2, slots=1, length=4096, positions=4096)
    e = fake_engine(s, 1)
    classes = select.gemv_classes(e)
    # q/k/v as one GEMV, o, [gate; up] interleaved, down, the LM head
    assert classes == [(12288, 4096, 1), (4096, 4096, 1), (22016, 4096, 1), (4096, 11008, 1), (32000, 4096, 1)]
    picks = [2, 1, 4, 8, 1]
    text = H.gemv_selection_render(classes, picks, 148)
    e.splits = select.splits_for(e, text)
    assert e.splits == {(n, k): p for (n, k, _), p in zip(classes, picks)}
    got, want = e._launches(), RL.decode_launches(e)
    assert [(L.kernel, L.params, L.bufs) for L in got] == [(L.kernel, L.params, L.bufs) for L in want]
    assert {(L.params["n"], L.params["k"]): L.params["split"] for L in got if L.kernel.startswith("gemv")} == \
        e.splits


def test_a_selection_for_other_classes_is_refused():
    from furykernel_b200 import select
    from furykernel_b200.shape import LlamaShape
    from tests.test_host_cpp import fake_engine

    e = fake_engine(LlamaShape(layers=1, slots=4, length=64, positions=64), 4)
    other = H.gemv_selection_render([(4096, 4096, 1)], [1], 148)
    with pytest.raises(N.Refused, match="No variant for the class n12288_k4096_m4"):
        select.splits_for(e, other)


def test_row_pair_kernels_take_split_one_past_batch_four():
    from furykernel_b200.shape import LlamaShape
    from tests.test_host_cpp import fake_engine

    e = fake_engine(LlamaShape(layers=1, slots=8, length=64, positions=64), 8)
    e.splits = {(22016, 4096): 2}
    with pytest.raises(N.Refused, match="row-pair kernels take split 1 past batch 4, not 2"):
        e._launches()
    with pytest.raises(N.Refused, match="row-pair kernels take split 1 past batch 4, not 2"):
        RL.decode_launches(e)


def test_tuning_picks_the_split_fastest_over_every_batch():
    from furykernel_b200 import select

    classes = [(4096, 11008, 1), (4096, 11008, 16), (4096, 4096, 1)]
    times = {(4096, 11008, 1): {1: 0.030, 2: 0.028, 4: 0.029},
             (4096, 11008, 16): {1: 0.070, 2: 0.080},          # 4 not kept at this batch
             (4096, 4096, 1): {1: 0.012, 8: 0.011}}
    assert select.choose(classes, times) == [1, 1, 8]
    with pytest.raises(N.Refused, match="no split is kept at every batch"):
        select.choose([(1, 4, 1), (1, 4, 2)], {(1, 4, 1): {1: 1.0}, (1, 4, 2): {2: 1.0}})


def test_routed_gemvs_are_no_gemv_class():
    """A model of routed experts: its classes are the dense GEMVs' (the
    projections, the router, the head), never the routed GEMV's, whose `k`
    is the route's rank count."""
    import dataclasses

    from furykernel_b200 import select as S
    from tests.test_host_cpp import fake_engine, small

    e = fake_engine(dataclasses.replace(small(3), experts=8, top_k=2), 3)
    classes = S.gemv_classes(e)
    assert classes and all(k >= 256 for _, k, _ in classes)
    assert (8, 512, 3) in classes  # the router


def test_classes_for_a_shape_are_the_engines():
    """classes_for (no device) names the same GEMV classes as the engine's
    launch list at every batch form: streaming, batched, chunked."""
    from furykernel_b200 import select as S
    from tests.test_host_cpp import fake_engine, small

    for b in (1, 5, 80):
        e = fake_engine(small(b), b)
        assert S.classes_for(small(b), b, 148) == S.gemv_classes(e)
    S.main(["classes", "--batches", "1,16", "--layers", "1"])


def test_the_committed_b200_selection_validates_for_config_5():
    """The selection tuned on a B200 (python -m furykernel_b200.select tune,
    148 SMs) for config 5's GEMV classes at batches 1, 4, 16 and 64 reads
    back against the current kernels' identities and picks, for every
    class, the split the engine takes by default (1)."""
    import os

    from furykernel_b200 import select as S
    from furykernel_b200.shape import LlamaShape

    path = os.path.join(os.path.dirname(S.__file__), "selections", "config5_b200.json")
    text = open(path).read()
    classes = []
    for b in (1, 4, 16, 64):
        length = 4096 if b <= 4 else 640
        classes += S.classes_for(LlamaShape(slots=b, length=length, positions=length), b, 148)
    assert H.gemv_selection_validate(text, classes, 148) == [1] * len(classes)
