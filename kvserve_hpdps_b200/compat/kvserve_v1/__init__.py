"""Alias package: the reference's module paths (kvserve_v1/...) served by
``kvserve_hpdps_b200``.

Importing ``kvserve_v1`` installs a finder for ``kvserve_v1.<sub>`` names.
Each alias module is a new module object whose public names are the same
objects as in the target module(s) (classes compare identical, so
``isinstance`` checks hold across both names); any other attribute is looked
up in the targets on access.  ``_RENAMES`` covers the reference names that
this package spells differently.
"""

from __future__ import annotations

import importlib
import importlib.abc
import importlib.machinery
import sys
import types

_P = "kvserve_hpdps_b200."

# alias (below kvserve_v1.) -> target modules, searched in order
_ALIASES: dict[str, tuple[str, ...]] = {
    "connector": ("connector.compressed_kv_connector",),
    "connector.compressed_kv_connector": ("connector.compressed_kv_connector",),
    "compression": ("compression",),
    "compression.manager": ("compression.manager",),
    "compression.wire": ("compression.wire",),
    "compression.components": ("compression.components",),
    "compression.compression_manager": ("compression.pipeline_manager", "compression.config"),
    "compression.tilelang_manager": ("compression.fused_manager",),
    "compression.codec": ("compression.codec",),
    "compression.codec.kvserve_codec": ("compression.codec",),
    "compression.codec.lc_codec": ("compression.codec",),
    "compression.codec.nvcomp_func": ("compression.codec",),
    "compression.quantizer": ("compression.quantizer", "compression.split"),
    "compression.quantizer.kvserve_quantizer": ("compression.quantizer",),
    "compression.quantizer.quantizer_func": ("compression.quantizer",),
    "compression.quantizer.split_func": ("compression.split",),
    "compression.transformer": ("compression.transformer",),
    "compression.transformer.kvserve_transformer": ("compression.transformer",),
    "compression.transformer.hadamard_func": ("compression.transformer",),
    "compression.controller": ("controller",),
    "compression.controller.profile": ("controller.profile",),
    "compression.controller.analytical_model": ("controller.analytical_model",),
    "compression.controller.bandit_state": ("controller.bandit_state",),
    "compression.controller.profile_library": ("controller.profile_library",),
    "compression.controller.online_controller": ("controller.online_controller",),
    "compression.config": ("compression.config",),
    "compression.config.duo_config": ("compression.head_scores",),
    "compression.config.duo_config.get_config": ("compression.head_scores",),
    "transport": ("parallel",),
    "transport.nccl_transport": ("parallel.nccl_transport",),
    "transport.zmq_transport": ("parallel.zmq_transport",),
    "utils": ("utils",),
    "utils.kv_utils": ("utils.kv_utils",),
    "utils.logger": ("utils.logger",),
    "tilelang_ops": ("ops.hadamard_quant_op",),
    "tilelang_ops.kv_hadamard_quant": ("ops.hadamard_quant_op",),
    "offline_search": ("offline",),
    "offline_search.src": ("offline.caches",),
    "offline_search.src.cache": ("offline.caches",),
    "offline_search.src.cache.cache_utils": ("offline.caches",),
    "offline_search.src.cache.kivi_utils": ("offline.caches",),
    "offline_search.src.cache.cachegen_utils": ("offline.caches",),
    "offline_search.src.cache.duoattn_utils": ("offline.caches",),
    "offline_search.duo_config": ("offline.duo_scores",),
    "offline_search.duo_config.duo_config": ("offline.duo_scores",),
    "offline_search.evaluation": ("offline",),
    "offline_search.evaluation.param_search": ("offline.param_search",),
    "offline_search.evaluation.param_search.acc_evaluator": ("offline.param_search",),
    "offline_search.evaluation.param_search.cr_evaluator": ("offline.param_search",),
    "offline_search.evaluation.lm_eval": ("offline.lm_harness",),
    "offline_search.evaluation.lm_eval.lm_wrapper": ("offline.lm_harness",),
}

# reference name -> name in the target modules
_RENAMES = {"TileLangCompressionManager": "FusedCompressionManager"}

# names that differ only under one alias (the offline Hadamard of the reference's
# cache_utils is this package's HeadHadamard; compression.transformer keeps its own)
_ALIAS_RENAMES: dict[str, dict[str, str]] = {
    "offline_search.src.cache.cache_utils": {"HadamardTransform": "HeadHadamard"},
    "offline_search.duo_config": {"duo_attention_on_the_fly": "duo_scores_on_the_fly"},
    "offline_search.duo_config.duo_config": {"duo_attention_on_the_fly": "duo_scores_on_the_fly"},
}

# aliases that have submodules (get a __path__)
_PACKAGES = {a.rsplit(".", 1)[0] for a in _ALIASES if "." in a}


def _resolve(targets: tuple[str, ...], name: str, renames: dict = _RENAMES):
    real = renames.get(name, name)
    for t in targets:
        mod = importlib.import_module(_P + t)
        if hasattr(mod, real):
            return getattr(mod, real)
    raise AttributeError(name)


class _AliasLoader(importlib.abc.Loader):
    def __init__(self, alias: str):
        self.alias = alias
        self.targets = _ALIASES[alias]

    def create_module(self, spec):
        return None  # default module object

    def exec_module(self, module: types.ModuleType) -> None:
        targets = self.targets
        names: list[str] = []
        for t in targets:
            mod = importlib.import_module(_P + t)
            pub = getattr(mod, "__all__", None)
            if pub is None:
                pub = [n for n in vars(mod) if not n.startswith("_")]
            for n in pub:
                if n not in names and hasattr(mod, n):
                    names.append(n)
                    setattr(module, n, getattr(mod, n))
        renames = {**_RENAMES, **_ALIAS_RENAMES.get(self.alias, {})}
        for ref_name, real in renames.items():
            for t in targets:
                mod = importlib.import_module(_P + t)
                if hasattr(mod, real):
                    setattr(module, ref_name, getattr(mod, real))
                    names.append(ref_name)
                    break
        module.__all__ = names
        module.__getattr__ = lambda name: _resolve(targets, name, renames)
        module.__doc__ = f"Alias of {', '.join(_P + t for t in targets)}."


class _AliasFinder(importlib.abc.MetaPathFinder):
    def find_spec(self, fullname, path=None, target=None):
        if not fullname.startswith("kvserve_v1."):
            return None
        alias = fullname[len("kvserve_v1."):]
        if alias not in _ALIASES:
            return None
        return importlib.machinery.ModuleSpec(fullname, _AliasLoader(alias),
                                              is_package=alias in _PACKAGES)


if not any(isinstance(f, _AliasFinder) for f in sys.meta_path):
    sys.meta_path.insert(0, _AliasFinder())

__all__ = ["CompressedKVConnector"]


def __getattr__(name):
    if name == "CompressedKVConnector":
        from kvserve_hpdps_b200.connector.compressed_kv_connector import CompressedKVConnector
        return CompressedKVConnector
    raise AttributeError(name)
