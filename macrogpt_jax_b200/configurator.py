"""`@config` / `.override()` factory injection, the mechanism macrogpt-jax uses to swap the
layers a module builds (ueaj/utils/configurator.py:69-161).  It is how the FP8 Einsum is
plugged in, e.g. ``GMLP.override(fused_proj=Einsum, down_proj=Einsum)``.

Behaviour kept from the reference (pinned by tests/test_reference_golden.py against the
reference's own configurator):
  * ``@config`` on a class or function adds ``.override(**kw)``, which returns a new
    configurable factory function; ``.override`` chains, later keys winning;
  * functions: an override replaces the argument whatever the caller passes at call time;
    ``override(**kw)`` as a value overrides the arguments of the current value of that
    parameter (``.override`` when it has one, ``functools.partial`` otherwise); an unknown key
    raises TypeError unless the function takes ``**kwargs``, where it is forwarded through them;
  * classes: the factory is ``lambda *args, **kwargs: Class(*args, **kwargs)``, so every
    override is forwarded as a constructor keyword (winning over a call-site keyword of the
    same name; a positional argument for the same parameter is an error of the constructor
    call), nothing is validated before construction, and a nested ``override(**kw)`` value is
    forwarded as it is.
"""
from __future__ import annotations

import functools
import inspect
from typing import Callable

_NESTED = "override"


def override(**kwargs) -> tuple:
    """Marks a value as 'override these arguments of the parameter's current value'."""
    return (_NESTED, kwargs)


def _is_nested(value) -> bool:
    return isinstance(value, tuple) and len(value) == 2 and value[0] == _NESTED and isinstance(value[1], dict)


def _var_kw_name(sig: inspect.Signature) -> str | None:
    for p in sig.parameters.values():
        if p.kind is inspect.Parameter.VAR_KEYWORD:
            return p.name
    return None


def _check_keys(name: str, sig: inspect.Signature, keys) -> None:
    if _var_kw_name(sig) is not None:
        return
    unknown = [k for k in keys if k not in sig.parameters]
    if unknown:
        allowed = [k for k in sig.parameters if k != "self"]
        raise TypeError(f"Invalid override {unknown[0]!r} for {name!r}. Available parameters: {allowed}")


def _call_with(target: Callable, sig: inspect.Signature, overrides: dict, args, kwargs):
    bound = sig.bind_partial(*args, **kwargs)
    bound.apply_defaults()
    var_kw = _var_kw_name(sig)
    for key, value in overrides.items():
        if key in sig.parameters and sig.parameters[key].kind is not inspect.Parameter.VAR_KEYWORD:
            if _is_nested(value):
                current = bound.arguments.get(key, sig.parameters[key].default)
                if hasattr(current, "override"):
                    bound.arguments[key] = current.override(**value[1])
                elif callable(current) and current is not inspect.Parameter.empty:
                    bound.arguments[key] = functools.partial(current, **value[1])
                else:
                    raise TypeError(f"Argument {key!r} is not configurable or callable; cannot override its arguments.")
            else:
                bound.arguments[key] = value
        elif var_kw is not None:
            bound.arguments.setdefault(var_kw, {})[key] = value
    return target(*bound.args, **bound.kwargs)


def _make_overridden(target: Callable, sig: inspect.Signature, name: str, overrides: dict):
    @functools.wraps(target)
    def factory(*args, **kwargs):
        return _call_with(target, sig, overrides, args, kwargs)

    factory.overrides = dict(overrides)

    def more(**kw):
        _check_keys(name, sig, kw)
        return _make_overridden(target, sig, name, {**overrides, **kw})

    factory.override = more
    return factory


def config(obj):
    """Adds ``.override(**kw)`` to a class or function (see module docstring)."""
    if inspect.isclass(obj):
        def construct(*args, **kwargs):
            return obj(*args, **kwargs)

        sig = inspect.signature(construct)  # (*args, **kwargs): every override is a keyword

        def cls_override(**kw):
            return _make_overridden(construct, sig, obj.__name__, kw)

        obj.override = staticmethod(cls_override)
        return obj
    if callable(obj):
        sig = inspect.signature(obj)
        name = getattr(obj, "__name__", repr(obj))

        def fn_override(**kw):
            _check_keys(name, sig, kw)
            return _make_overridden(obj, sig, name, kw)

        obj.override = fn_override
        return obj
    raise TypeError("@config can only be used on callables (functions or classes)")


__all__ = ["config", "override"]
