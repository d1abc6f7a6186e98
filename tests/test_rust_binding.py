"""The Rust binding (rust/ammon-b200-sys, rust/ammon-b200) against the C header, on CPU: there
is no Rust toolchain in this image, so the sources are checked by parsing. Every function the
header declares has an extern "C" declaration with the same number of parameters (and no extra
ones), the #[repr(C)] structs list the header's fields in order, and the safe crate exports the
reference crate's public names (src/lib.rs re-exports)."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    src = open(os.path.join(ROOT, "include", "ammon_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for ret, name, args in re.findall(r"^\s*((?:const\s+)?[\w\s\*]+?)\s*\b(ab_\w+)\s*\(([^;{]*?)\)\s*;",
                                      src, flags=re.M):
        a = args.strip()
        out[name] = 0 if a in ("", "void") else len(a.split(","))
    return out, src


def _rust_functions():
    src = open(os.path.join(ROOT, "rust", "ammon-b200-sys", "src", "lib.rs")).read()
    out = {}
    for name, args in re.findall(r"pub fn (ab_\w+)\(([^)]*)\)", src):
        a = args.strip()
        out[name] = 0 if not a else len(a.split(","))
    return out, src


def test_every_header_function_is_declared_with_its_arity():
    h, _ = _header_functions()
    r, _ = _rust_functions()
    assert len(h) > 80
    assert set(h) == set(r), (sorted(set(h) - set(r)), sorted(set(r) - set(h)))
    assert {k: v for k, v in h.items() if r[k] != v} == {}


def _c_struct_fields(src, name):
    body = re.search(r"typedef struct\s*\{([^{}]*)\}\s*" + name + r"\s*;", src).group(1)
    fields = []
    for decl in body.split(";"):
        decl = " ".join(decl.split())
        if not decl:
            continue
        fn = re.search(r"\(\*(\w+)\)", decl)
        if fn:  # a function pointer member
            fields.append(fn.group(1))
            continue
        names = decl.replace("*", " ").split(None, 1)[1]  # drop the type
        fields += [re.sub(r"\[.*\]", "", n).strip() for n in names.split(",")]
    return fields


def _rust_struct_fields(src, name):
    m = re.search(r"pub struct " + name + r"\s*\{(.*?)\}", src, flags=re.S)
    return re.findall(r"pub (\w+):", m.group(1))


def test_repr_c_structs_follow_the_header():
    _, hsrc = _header_functions()
    _, rsrc = _rust_functions()
    for name in ("ab_tensor", "ab_decode_step", "ab_llama_config", "ab_attention_weights",
                 "ab_swiglu_weights"):
        assert _c_struct_fields(hsrc, name) == _rust_struct_fields(rsrc, name), name
    # the vtable's first member is `self` in C (a Rust keyword: self_)
    want = ["self_" if f == "self" else f for f in _c_struct_fields(hsrc, "ab_autoregressive_model")]
    assert _rust_struct_fields(rsrc, "ab_autoregressive_model") == want


def test_safe_crate_exports_the_reference_names():
    src = open(os.path.join(ROOT, "rust", "ammon-b200", "src", "lib.rs")).read()
    for name in ("Embedding", "RmsNorm", "Linear", "CausalAttentionBlock",
                 "CausalAttentionBlockWeights", "SwiGluBlock", "SwiGluBlockWeights", "KvCache",
                 "KvLayer", "DecodeStep", "BpeTokenizer"):
        assert re.search(r"pub struct " + name + r"\b", src), name
    for name in ("AutoregressiveModel", "Tokenizer"):
        assert re.search(r"pub trait " + name + r"\b", src), name
    for name in ("generate_tokens", "sample_argmax"):
        assert re.search(r"pub fn " + name + r"\b", src), name
    # every sys call the safe crate makes exists
    r, _ = _rust_functions()
    for call in set(re.findall(r"sys::(ab_\w+)\(", src)):
        assert call in r, call
