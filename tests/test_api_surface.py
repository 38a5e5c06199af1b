"""The drop-in surface: every reference name this package replaces, with the reference's members and signatures.

A user switches ``from anchorkv.backend / .policy / .packed_decode /
.triton_decode import ...`` to ``from anchorkv_b200 import ...``.  For each
replaced function and type, this compares against the reference installed
unmodified in baseline/_ref: the name exists, a type has every public member
the reference's has, and every callable takes the reference's parameters
(names, kinds and defaults, in order; extra trailing keyword-only parameters
are allowed).
"""

import inspect
import pytest

import anchorkv_b200 as akv

REPLACED = {
    "backend": ["quantize_tensor", "PackedTensor", "DeclarativeKVCache", "SegmentRole", "AttentionMode",
                "DirectiveKind", "CacheDirective", "DeclarativeAttentionParser", "DeclarativeState",
                "LossyPromotionError", "BackendUnavailableError", "stack_legacy_cache", "KVBlock",
                "SegmentRecord", "MaterializedCache"],
    "policy": ["CacheMode", "CachePlan", "PlannedSegment"],
    "packed_decode": ["PagedLayer", "pack_page", "QuantizedPage", "dense_attention", "kl_divergence",
                      "tensor_bytes"],
    "triton_decode": ["packed_attention"],
    "heads": ["query_head_to_kv_head"],
}


@pytest.fixture(scope="module")
def reference(reference_install):
    import importlib

    return {name: importlib.import_module(f"anchorkv.{name}") for name in REPLACED}


def _default(value):
    # a dataclass field with a default factory shows a sentinel; a None default that builds a
    # fresh object in __init__ means the same to a caller
    return None if repr(value) == "<factory>" else value


def _params(fn):
    try:
        return [(p.name, p.kind, _default(p.default)) for p in inspect.signature(fn).parameters.values()]
    except (TypeError, ValueError):  # builtins without a signature
        return None


def _same_parameters(ref_fn, our_fn, what):
    ref, ours = _params(ref_fn), _params(our_fn)
    if ref is None or ours is None:
        return
    extra = ours[len(ref):]
    assert ours[:len(ref)] == ref, f"{what}: {ref} != {ours}"
    assert all(kind is inspect.Parameter.KEYWORD_ONLY for _, kind, _ in extra), f"{what}: extra {extra}"


@pytest.mark.parametrize("module,name", [(m, n) for m, names in REPLACED.items() for n in names])
def test_replaced_names_keep_the_reference_surface(reference, module, name):
    ref_obj = getattr(reference[module], name)
    assert hasattr(akv, name), f"anchorkv_b200 lacks {name}"
    ours = getattr(akv, name)
    if not inspect.isclass(ref_obj):
        _same_parameters(ref_obj, ours, name)
        return
    ref_members = {m for m in dir(ref_obj) if not m.startswith("_")}
    missing = ref_members - {m for m in dir(ours) if not m.startswith("_")}
    assert not missing, f"{name} lacks {sorted(missing)}"
    if issubclass(ref_obj, BaseException):
        assert issubclass(ours, tuple(b for b in ref_obj.__mro__[1:] if b.__module__ == "builtins"))
    if not issubclass(ref_obj, (BaseException,)) and not hasattr(ref_obj, "__members__"):
        _same_parameters(ref_obj, ours, name)  # constructor
    if hasattr(ref_obj, "__members__"):  # an enum: the same members with the same values
        assert {k: v.value for k, v in ref_obj.__members__.items()} == \
            {k: v.value for k, v in ours.__members__.items()}
    for member in ref_members:
        a, b = getattr(ref_obj, member), getattr(ours, member)
        if callable(a) and not inspect.isclass(a):
            _same_parameters(a, b, f"{name}.{member}")
