"""Fixed EAGLE3 draft trees (``llmserve/speculative/tree.py`` of the reference).

Topologies with 6 or 10 draft nodes given by parent tuples, the ancestor attention mask, and
greedy path selection (walk from the root, following the child whose draft token equals the
target argmax at the current node).
"""
from dataclasses import dataclass

import torch


@dataclass(frozen=True, slots=True)
class Eagle3TreeTopology:
    parents: tuple[int, ...]

    def __post_init__(self):
        if not self.parents or self.parents[0] != -1:
            raise ValueError("tree root must have parent -1")
        for i, p in enumerate(self.parents[1:], start=1):
            if p < 0 or p >= i:
                raise ValueError("tree parents must precede their children")

    @property
    def num_draft_nodes(self) -> int:
        return len(self.parents) - 1

    @property
    def depths(self) -> tuple[int, ...]:
        d = [0]
        for p in self.parents[1:]:
            d.append(d[p] + 1)
        return tuple(d)

    def children(self, node: int) -> tuple[int, ...]:
        return tuple(i for i, p in enumerate(self.parents) if p == node)

    def ancestors_and_self(self, node: int) -> list[int]:
        out = []
        while node >= 0:
            out.append(node)
            node = self.parents[node]
        return out

    def attention_mask(self, device=None) -> torch.Tensor:
        n = len(self.parents)
        mask = torch.zeros((n, n), dtype=torch.bool)
        for i in range(n):
            for a in self.ancestors_and_self(i):
                mask[i, a] = True
        return mask.to(device) if device is not None else mask


@dataclass(slots=True)
class Eagle3TreeAcceptResult:
    token_ids: list[int]
    accepted_node_indices: list[int]
    commit_node_indices: list[int]
    final_token_id: int
    final_node_index: int
    num_accepted: int
    accepted_all: bool


def build_fixed_tree_topology(num_draft_nodes: int) -> Eagle3TreeTopology:
    table = {6: (-1, 0, 0, 1, 2, 3, 4), 10: (-1, 0, 0, 1, 1, 2, 2, 3, 4, 5, 6)}
    if num_draft_nodes not in table:
        raise ValueError("fixed EAGLE3 tree supports 6 or 10 draft nodes")
    return Eagle3TreeTopology(table[num_draft_nodes])


def select_greedy_tree_path(topology: Eagle3TreeTopology, draft_token_ids: list[int],
                            target_argmax: list[int]) -> Eagle3TreeAcceptResult:
    if len(draft_token_ids) != topology.num_draft_nodes:
        raise ValueError("draft token count does not match tree topology")
    if len(target_argmax) != len(topology.parents):
        raise ValueError("target logits do not match tree topology")
    node, accepted, tokens = 0, [], []
    while True:
        want = int(target_argmax[node])
        nxt = next((c for c in topology.children(node) if int(draft_token_ids[c - 1]) == want), None)
        if nxt is None:
            final = want
            break
        accepted.append(nxt)
        tokens.append(want)
        node = nxt
    return Eagle3TreeAcceptResult(tokens + [final], accepted, [0] + accepted, final, node, len(accepted),
                                  not topology.children(node))
