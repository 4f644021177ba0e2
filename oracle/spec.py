"""Oracle: speculation bookkeeping (CPU, TEST INFRASTRUCTURE ONLY).

Plain-Python restatements, row by row, of the reference's fused bookkeeping kernels:
  engine/kernels/spec.py:16-124   `_propose` / `propose`       (drafting one verify block)
  engine/kernels/spec.py:127-166  `_within_margin`             (relaxed acceptance flags)
  engine/kernels/spec.py:169-240  `_settle` / `settle`         (accept, emit, plan the KV move)
  engine/kernels/spec.py:243-270  `_relocate` / `relocate`     (move one K/V slot per row)
Pinned against fixtures the reference's own wrappers produced (tests/golden/spec.pt).
"""

import torch


def _matches(h, place, size, maxlen):
    """Occurrences of the newest token h[place] before `place`, each ranked by how long a
    suffix ending there agrees with the suffix ending at `place` (up to maxlen tokens):
    rank = index + (length - 1) * size, -1 for non-occurrences (spec.py:38-49)."""
    last = h[place]
    rank = [-1] * size
    for i in range(size):
        if not (i < place and h[i] == last):
            continue
        length = 1
        for back in range(1, maxlen):
            if i < back or place < back or h[i - back] != h[max(place - back, 0)]:
                break
            length += 1
        rank[i] = i + (length - 1) * size
    return rank


def propose_row(h, place, successor, size, tokens, drafts_by_match, maxlen, stale):
    """One row of spec.py:_propose: (tokens, chain length, RoPE phases)."""
    top = len(successor[0])
    lanes = tokens - 1 - min(drafts_by_match)
    last = h[place]
    rank = _matches(h, place, size, maxlen)
    best = max(rank)
    found = best >= 0
    start = best % size if found else place
    matched = best // size + 1 if found else 0
    d0, d1, d2, d3 = drafts_by_match
    drafts = d0 if matched <= 1 else d1 if matched <= 3 else d2 if matched <= 7 else d3
    out = [0] * tokens
    out[0] = last
    previous, first = last, last
    for step in range(1, tokens):
        source = start + step
        draft = h[min(source, size - 1)] if (found and source <= place) else successor[previous][0]
        if step <= drafts:
            out[step] = draft
        previous = draft
        if step == 1:
            first = draft
    if lanes > 0:
        siblings, count = [], 0
        if stale >= 0 and stale != first and tokens - 1 - drafts >= 2:
            siblings.append(stale)
            count = 1
        # what followed other occurrences of the newest token, longest agreement first
        after = [h[i + 1] if rank[i] >= 0 else -1 for i in range(size)]
        for _ in range(min(lanes, 3)):
            open_ranks = [rank[i] for i in range(size)
                          if rank[i] >= 0 and after[i] != first and after[i] not in siblings]
            choice = max(open_ranks) if open_ranks else -1
            if choice >= 0 and count < lanes:
                siblings.append(h[choice % size + 1])
                count += 1
        # then the successor table's choices after the newest token
        for entry in range(top):
            candidate = successor[last][entry]
            if candidate != first and candidate not in siblings and count < lanes:
                siblings.append(candidate)
                count += 1
        for lane in range(lanes):
            if 1 + drafts + lane < tokens:
                out[1 + drafts + lane] = siblings[lane] if lane < len(siblings) else first
    phases = [slot if slot <= drafts else 1 for slot in range(tokens)]
    return out, 1 + drafts, phases


def propose(history, position, tokens_per_row, drafts_by_match, successor, stale, maxlen=8):
    """spec.py:106-124 over every row: (tokens [B, T], chains [B], phases [B, T]) int64."""
    batch, size = history.shape
    table = successor.tolist()
    out, chains, phases = [], [], []
    for b in range(batch):
        row, chain, phase = propose_row(history[b].tolist(), int(position[b]), table, size, tokens_per_row,
                                        tuple(drafts_by_match), maxlen, int(stale[b]))
        out.append(row)
        chains.append(chain)
        phases.append(phase)
    return (torch.tensor(out, dtype=torch.int64), torch.tensor(chains, dtype=torch.int64),
            torch.tensor(phases, dtype=torch.int64))


def within_margin(logits, tokens, top, margin):
    """spec.py:127-151: flag [B, T] whether draft `slot` (>= 1) sits within `margin` of the
    winning logit of the row that produced it (slot - 1). Slot 0 is not a draft: 0 here."""
    batch, count = tokens.shape
    values = logits.float()
    bound = top.view(-1).float() - torch.tensor(margin, dtype=torch.float32)  # fp32, as the kernel
    flags = torch.zeros(batch, count, dtype=torch.int64)
    for b in range(batch):
        for slot in range(1, count):
            previous = b * count + slot - 1
            flags[b, slot] = int(bool(values[previous, int(tokens[b, slot])] >= bound[previous]))
    return flags


def settle(tokens, greedy, position, limit, history, chains, stale, within=None):
    """spec.py:169-240, returning (result [B, T+1], history, move_from, move_to, position,
    stale) as new tensors: keep the chain drafts up to the first illegal one, or branch to an
    alternative equal to the model's first choice; clamp at `limit`; emit what was in context."""
    batch, count = tokens.shape
    history, position, stale = history.clone(), position.clone(), stale.clone()
    result = torch.zeros(batch, count + 1, dtype=torch.int64)
    move_from = torch.zeros(batch, dtype=torch.int64)
    move_to = torch.zeros(batch, dtype=torch.int64)
    for b in range(batch):
        chain = int(chains[b])
        draft, chosen = tokens[b].tolist(), greedy[b].tolist()
        if within is None:
            legal = [slot >= 1 and draft[slot] == chosen[slot - 1] for slot in range(count)]
        else:
            legal = [bool(within[b, slot]) for slot in range(count)]
        gained = chain
        for slot in range(1, min(chain, count)):
            if not legal[slot]:
                gained = slot
                break
        accepted = gained
        hit = next((slot for slot in range(chain, count) if draft[slot] == chosen[0]), count)
        place = int(position[b])
        room = max(int(limit[b]) - place, 0)
        branch = gained == 1 and hit < count and room >= 2
        stale[b] = chosen[min(gained, count - 1)] if (gained < chain and not branch) else -1
        gained = min(2 if branch else gained, room)
        emitted = [draft[slot + 1] if (slot + 1 < accepted and slot + 1 < count) else chosen[slot]
                   for slot in range(count)]
        if branch:
            emitted[1] = chosen[min(hit, count - 1)]
        result[b, 0] = gained
        result[b, 1:] = torch.tensor(emitted, dtype=torch.int64)
        history[b, place + 1:place + 1 + count] = torch.tensor(emitted, dtype=torch.int64)
        move_from[b] = place + hit if branch else -1
        move_to[b] = place + 1
        position[b] = place + gained
    return result, history, move_from, move_to, position, stale


def relocate(store, move_from, move_to):
    """spec.py:243-270: in every (K/V, layer) plane, row b's slot move_from[b] is copied to
    move_to[b] (all heads), where move_from[b] >= 0. Returns the moved store."""
    moved = store.clone()
    for b in range(store.shape[2]):
        source, target = int(move_from[b]), int(move_to[b])
        if source >= 0:
            moved[:, :, b, :, target] = store[:, :, b, :, source]
    return moved
