"""Implementation registry with the plugin API of kapitan05/ace-kernels.

Code written against ``ace_kernels.registry`` (``src/ace_kernels/registry.py``
there) keeps working here: the same five names exist with the same arguments,
and the same error types are raised (``ValueError`` for a name taken twice or an
unsupported binning/device, ``KeyError`` for an unknown name). Entries live in a
:class:`Registry`; the module-level functions act on the package's default one,
where ``ace_kernels_b200`` registers ``b200_cuda`` at import. (When the reference
package is importable, ``ace_kernels_b200.plugin`` also enters ``b200_cuda`` in
the reference's own registry.)
"""

from __future__ import annotations

from collections.abc import Callable, Iterator
from dataclasses import dataclass, field

import torch

from ace_kernels_b200.config import ACEConfig, Binning

ACEFn = Callable[[torch.Tensor, torch.Tensor, ACEConfig], torch.Tensor]

ALL_BINNINGS: frozenset[Binning] = frozenset({"hard", "soft"})
ALL_DEVICES: frozenset[str] = frozenset({"cpu", "cuda"})


@dataclass(frozen=True)
class ImplSpec:
    """One loss implementation: its callable ``fn(input, target, config)`` and
    the binnings and device types it accepts (``slow``: excluded from heavy test
    and benchmark sweeps)."""

    name: str
    fn: ACEFn
    binnings: frozenset[Binning]
    devices: frozenset[str]
    description: str
    slow: bool = False

    def supports(self, binning: Binning, device: str) -> bool:
        return binning in self.binnings and device in self.devices


@dataclass
class Registry:
    """Name -> :class:`ImplSpec` table with registration, lookup and dispatch."""

    entries: dict[str, ImplSpec] = field(default_factory=dict)

    def add(self, spec: ImplSpec) -> None:
        if spec.name in self.entries:
            raise ValueError(f"an implementation named {spec.name!r} exists already")
        self.entries[spec.name] = spec

    def lookup(self, name: str) -> ImplSpec:
        spec = self.entries.get(name)
        if spec is None:
            known = ", ".join(sorted(self.entries)) or "none"
            raise KeyError(f"no implementation named {name!r} (registered: {known})")
        return spec

    def select(self, binning: Binning | None, device: str | None) -> list[ImplSpec]:
        return [s for s in self if (binning is None or binning in s.binnings)
                and (device is None or device in s.devices)]

    def dispatch(self, name: str, input: torch.Tensor, target: torch.Tensor,
                 config: ACEConfig) -> torch.Tensor:
        spec = self.lookup(name)
        device = input.device.type
        if not spec.supports(config.binning, device):
            raise ValueError(
                f"implementation {name!r} cannot run {config.binning} binning on a "
                f"{device} tensor (it takes binnings {sorted(spec.binnings)} on "
                f"devices {sorted(spec.devices)})"
            )
        return spec.fn(input, target, config)

    def __iter__(self) -> Iterator[ImplSpec]:
        return iter(self.entries.values())


DEFAULT = Registry()
# the default registry's table (tests substitute entries through it)
_REGISTRY = DEFAULT.entries


def register(
    name: str,
    *,
    description: str,
    binnings: frozenset[Binning] = ALL_BINNINGS,
    devices: frozenset[str] = ALL_DEVICES,
    slow: bool = False,
) -> Callable[[ACEFn], ACEFn]:
    """Class-free decorator form of :meth:`Registry.add` on the default registry;
    returns the function unchanged."""

    def enter(fn: ACEFn) -> ACEFn:
        DEFAULT.add(ImplSpec(name, fn, frozenset(binnings), frozenset(devices), description, slow))
        return fn

    return enter


def get_impl(name: str) -> ImplSpec:
    return DEFAULT.lookup(name)


def available_impls(binning: Binning | None = None, device: str | None = None) -> list[ImplSpec]:
    """Implementations of the default registry accepting ``binning`` and
    ``device`` (either filter may be left out)."""
    return DEFAULT.select(binning, device)


def ace_loss(
    input: torch.Tensor,
    target: torch.Tensor,
    config: ACEConfig | None = None,
    impl: str = "b200_cuda",
) -> torch.Tensor:
    """mL1-ACE of ``input`` (``[B, C, *spatial]`` logits, or probabilities when
    the config's activation is "none") against ``target`` (``[B, C, ...]``
    targets, or ``[B, 1, ...]`` class indices with ``to_onehot_y``), computed by
    the implementation registered as ``impl``; ``config`` defaults to
    ``ACEConfig()``."""
    return DEFAULT.dispatch(impl, input, target, config if config is not None else ACEConfig())
