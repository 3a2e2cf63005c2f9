"""Topology: worker name -> {host, layers}, as DIAL's topology.yml
(dial-core/src/spm/topology.rs:9-123), mapped onto pipeline stages.

Inside one 8xB200 box each node becomes one stage on its own GPU; the
stage order is the order of the nodes' first layers.
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field

import yaml

_RANGE = re.compile(r"^(.+[^\d])(\d+)-(\d+)$", re.M)


class TopologyError(ValueError):
    pass


@dataclass
class Node:
    host: str
    layers: list[str]
    description: str | None = None

    def is_layer_owner(self, full_layer_name: str) -> bool:
        """Node::is_layer_owner (topology.rs:24-31): prefix match on 'prefix.'."""
        return any(full_layer_name.startswith(p + ".") for p in self.layers)


def expand_layers(names: list[str]) -> list[str]:
    """Range expressions 'prefix.N-M' expand to N..=M (topology.rs:54-95)."""
    out: list[str] = []
    for name in names:
        m = _RANGE.match(name)
        if m:
            base, start, stop = m.group(1), int(m.group(2)), int(m.group(3))
            if stop <= start:
                raise TopologyError(f"invalid range expression {name}, end must be > start")
            out.extend(f"{base}{n}" for n in range(start, stop + 1))
        else:
            out.append(name)
    return out


def _layer_index(name: str) -> int:
    m = re.search(r"(\d+)$", name)
    if not m:
        raise TopologyError(f"layer name {name!r} has no index")
    return int(m.group(1))


@dataclass
class Topology:
    nodes: dict[str, Node] = field(default_factory=dict)

    @classmethod
    def from_yaml(cls, text: str) -> "Topology":
        raw = yaml.safe_load(text) or {}
        if not isinstance(raw, dict):
            raise TopologyError("topology must be a mapping of worker name -> node")
        nodes = {}
        for name, spec in raw.items():
            if not isinstance(spec, dict) or "host" not in spec or "layers" not in spec:
                raise TopologyError(f"node {name!r} needs 'host' and 'layers'")
            nodes[str(name)] = Node(host=str(spec["host"]), layers=expand_layers(list(spec["layers"])),
                                    description=spec.get("description"))
        return cls(nodes)

    @classmethod
    def from_path(cls, path: str) -> "Topology":
        with open(path) as f:
            return cls.from_yaml(f.read())

    @classmethod
    def even_split(cls, num_layers: int, n_stages: int, prefix: str = "model.layers.") -> "Topology":
        """Contiguous, as-even-as-possible split (earlier stages take the remainder)."""
        if n_stages < 1 or n_stages > num_layers:
            raise TopologyError(f"cannot split {num_layers} layers into {n_stages} stages")
        nodes, start = {}, 0
        for s in range(n_stages):
            n = num_layers // n_stages + (1 if s < num_layers % n_stages else 0)
            nodes[f"stage{s}"] = Node(host=f"cuda:{s}", layers=[f"{prefix}{i}" for i in range(start, start + n)])
            start += n
        return cls(nodes)

    def get_node_for_layer(self, layer_name: str):
        """topology.rs:98-109: exact match of an expanded layer name."""
        for name, node in self.nodes.items():
            if layer_name in node.layers:
                return name, node
        return None

    def stages(self, num_layers: int) -> list[tuple[str, int, int]]:
        """(node, first_layer, count) per stage, ordered by first layer; every node must
        own one contiguous range and together they must cover 0..num_layers-1 once."""
        ranges = []
        for name, node in self.nodes.items():
            idx = sorted(_layer_index(l) for l in node.layers)
            if not idx:
                continue
            if idx != list(range(idx[0], idx[0] + len(idx))):
                raise TopologyError(f"node {name!r} does not own one contiguous layer range")
            ranges.append((idx[0], len(idx), name))
        ranges.sort()
        covered = 0
        for first, count, name in ranges:
            if first != covered:
                raise TopologyError(f"layers {covered}..{first - 1} are not owned by any node")
            covered = first + count
        if ranges and covered != num_layers:
            raise TopologyError(f"topology covers {covered} of {num_layers} layers")
        return [(name, first, count) for first, count, name in ranges]
