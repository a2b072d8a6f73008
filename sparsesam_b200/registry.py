"""Algorithm registry — the reference's plugin API for SAM encoder patches.

Mirrors algos/registry.py of hchautran/SparseSAM: one `AlgoSpec` per
(backbone, name), `register()`, the generic `_apply` behind `apply_sam`,
`remove_all_sam` / `update_sam_ratio`, and the `_kw_sam_basic` /
`_bake_sam_apply` adapters. Only the SAM-backbone SparseSAM entries are
registered here (the other algorithms of the reference are outside this
package's scope); their patch is sparsesam_b200.sparsesam.sam.apply_patch.
"""
from __future__ import annotations

import inspect
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Tuple


@dataclass
class AlgoSpec:
    """One patch algorithm (algos/registry.py:20-31)."""
    name: str
    backbone: str                              # "sam" | "pe"
    apply: Callable[..., Any]
    kwargs_from_args: Optional[Callable[[Any, Optional[float]], dict]] = None
    accepts_ratio: bool = True
    category: str = "compress"                 # "compress" | "partial" | "attention"
    description: str = ""
    # SAM-only: classes used by `remove_all_sam` to revert subclassed modules.
    block_class: Optional[type] = None
    attn_class: Optional[type] = None


REGISTRY: Dict[Tuple[str, str], AlgoSpec] = {}

# Per-algorithm registration errors ("backbone:name" -> exception), as in the reference.
REGISTRATION_ERRORS: Dict[str, Exception] = {}


def register(spec: AlgoSpec) -> AlgoSpec:
    key = (spec.backbone, spec.name)
    if key in REGISTRY:
        raise ValueError(f"{spec.backbone} algorithm {spec.name!r} already registered")
    REGISTRY[key] = spec
    return spec


def specs_for(backbone: str) -> Dict[str, AlgoSpec]:
    return {n: s for (bb, n), s in REGISTRY.items() if bb == backbone}


def choices(backbone: str) -> List[str]:
    """Valid names for `backbone`, including the no-op 'none' baseline."""
    return ["none"] + sorted(specs_for(backbone).keys())


def spec_of(backbone: str, name: str) -> Optional[AlgoSpec]:
    return REGISTRY.get((backbone, name))


def _apply(model, backbone: str, name: str, args=None, ratio: Optional[float] = None, **extra):
    """Generic apply (algos/registry.py:61-82): 'none' and SAM ratio >= 1.0 are no-ops."""
    if name == "none":
        return None
    if backbone == "sam" and ratio is not None and ratio >= 1.0:
        return None
    spec = spec_of(backbone, name)
    if spec is None:
        raise KeyError(f"Unknown {backbone} algorithm {name!r}. Valid choices: {choices(backbone)}")
    if spec.kwargs_from_args is not None:
        kwargs = spec.kwargs_from_args(args, ratio)
    elif backbone == "sam":
        kwargs = dict(ratio=ratio)
    else:
        kwargs = {}
    kwargs.update(extra)
    return spec.apply(model, **kwargs)


def apply_sam(encoder, name, args=None, ratio=None, **extra):
    return _apply(encoder, "sam", name, args, ratio, **extra)


def sam_algo_choices() -> List[str]:
    return choices("sam")


def _safe_delattr(obj, *attrs):
    for a in attrs:
        if hasattr(obj, a):
            try:
                delattr(obj, a)
            except AttributeError:
                pass


def remove_all_sam(encoder, mask_decoder=None) -> int:
    """Idempotently undo every SAM patch (algos/registry.py:139-161): revert the
    subclassed Block/Attention modules, clear encoder.tome_info, instance-level
    forward overrides and the device weight caches. `mask_decoder` is accepted
    for API symmetry."""
    from .host import resolve_host
    _, Block, Attention = resolve_host()
    sam_specs = list(specs_for("sam").values())
    block_classes = tuple({s.block_class for s in sam_specs if s.block_class})
    attn_classes = tuple({s.attn_class for s in sam_specs if s.attn_class})
    n = 0
    for module in encoder.modules():
        t = type(module)
        if block_classes and t in block_classes:
            module.__class__ = Block
            n += 1
        elif attn_classes and t in attn_classes:
            module.__class__ = Attention
            n += 1
        for attr in ("_ssam_w", "_tome_info"):
            module.__dict__.pop(attr, None)
    _safe_delattr(encoder, "tome_info")
    encoder.__dict__.pop("forward", None)
    for blk in getattr(encoder, "blocks", []):
        blk.__dict__.pop("forward", None)
    return n


def update_sam_ratio(encoder, ratio: float):
    """Update the ratio without re-patching (works if already patched)."""
    if hasattr(encoder, "tome_info"):
        encoder.tome_info["ratio"] = ratio


def _kw_sam_basic(args, ratio):
    """(argparse.Namespace, ratio) -> apply kwargs (algos/registry.py:213-219)."""
    return dict(
        ratio=float(ratio if ratio is not None else args.ratios[0]),
        margin=float(getattr(args, "margin", 0.5)),
        mlp_merge=bool(getattr(args, "mlp_merge", True)),
        piecewise_block_size=int(getattr(args, "piecewise_block_size", 64)),
    )


def _bake_sam_apply(apply_fn, internal_algo: str):
    """Pre-bind `algo=internal_algo`; forward optional kwargs only when the patch
    signature accepts them (algos/registry.py:222-234)."""
    accepted = set(inspect.signature(apply_fn).parameters)

    def _apply_baked(encoder, ratio, margin=0.5, **extra):
        kw = dict(algo=internal_algo, ratio=ratio, margin=margin)
        for k, v in extra.items():
            if k in accepted:
                kw[k] = v
        return apply_fn(encoder, **kw)

    return _apply_baked


def _safe_register(backbone, name, make_spec):
    try:
        register(make_spec())
    except Exception as e:  # recorded, as in the reference
        REGISTRATION_ERRORS[f"{backbone}:{name}"] = e


def _register_sam():
    def _from_sparsesam():
        from .sparsesam.sam import ToMeSAMAttention as A
        from .sparsesam.sam import ToMeSAMBlock as B
        from .sparsesam.sam import apply_patch as fn
        return fn, B, A

    table = [
        ("sparsesam", _from_sparsesam, "tome", "SparseSAM Z-group merge on the SAM encoder (B200 kernels)."),
        ("sparsesam_pitome", _from_sparsesam, "pitome", "SparseSAM registered under its PiToMe alias."),
    ]
    for name, importer, internal_algo, desc in table:
        def mk(_imp=importer, _ia=internal_algo, _n=name, _d=desc):
            fn, B, A = _imp()
            return AlgoSpec(_n, "sam", _bake_sam_apply(fn, _ia), kwargs_from_args=_kw_sam_basic,
                            block_class=B, attn_class=A, description=_d)
        _safe_register("sam", name, mk)


_register_sam()

SAM_REGISTRY = specs_for("sam")

__all__ = [
    "AlgoSpec", "REGISTRY", "REGISTRATION_ERRORS", "register", "specs_for", "spec_of", "choices",
    "apply_sam", "remove_all_sam", "update_sam_ratio", "sam_algo_choices", "SAM_REGISTRY",
]
