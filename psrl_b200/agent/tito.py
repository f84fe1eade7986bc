"""Token-in / token-out (TITO) session records → training data (C26).

A session is a list of turns; each turn records the exact token ids the engine
received (``input_ids``, the whole context) and produced (``output_ids`` with
their log-probs).  The training sample is

* ``prompt_ids`` — the first turn's input;
* ``response_ids`` — everything after it: each turn's generated tokens (mask 1)
  followed by the tokens the environment/tools appended before the next turn
  (mask 0, log-prob 0);
* ``turn_count`` and, for MoE routed-expert replay, the concatenated per-token
  expert indices of generated tokens.

Reference: ``psrl/utils/tito/training_data.py:42``.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class TurnRecord:
    input_ids: list
    output_ids: list
    output_logprobs: list
    versions: list = field(default_factory=list)
    routed_experts: list | None = None


@dataclass
class TrainingSample:
    prompt_ids: list
    response_ids: list
    response_mask: list
    rollout_logprobs: list
    versions: list
    turn_count: int
    routed_experts: list | None = None


def build_training_data(turns: list[TurnRecord], final_obs: list | None = None) -> TrainingSample:
    if not turns:
        raise ValueError("empty session")
    prompt = list(turns[0].input_ids)
    resp, mask, lps, vers = [], [], [], []
    experts = [] if any(t.routed_experts is not None for t in turns) else None
    context = list(prompt)
    for i, t in enumerate(turns):
        if i > 0:
            if t.input_ids[: len(context)] != context:
                raise ValueError(f"turn {i} input does not extend the session context")
            env = t.input_ids[len(context):]
            resp += env
            mask += [0] * len(env)
            lps += [0.0] * len(env)
            vers += [-1] * len(env)
            context += env
        resp += t.output_ids
        mask += [1] * len(t.output_ids)
        lps += list(t.output_logprobs)
        vers += list(t.versions) if t.versions else [-1] * len(t.output_ids)
        if experts is not None:
            experts += list(t.routed_experts or [None] * len(t.output_ids))
        context += t.output_ids
    if final_obs:
        pass  # observations after the last turn are not part of the sample
    return TrainingSample(prompt, resp, mask, lps, vers, len(turns), experts)
