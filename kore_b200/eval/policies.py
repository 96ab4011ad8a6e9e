"""Policies that the evaluation harness can run on a task.

A policy maps a task to the list of candidate kernel sources it proposes
within its attempt budget (``evaluate_policy`` benches them and keeps the
best correct one). Three kinds:

* :func:`seed_policy`: the task's seed kernel (the floor every policy should
  clear);
* :func:`model_policy`: a chat model (our checkpoint through
  :class:`~kore_b200.data.teacher.LocalTeacher`, or any client with
  ``generate(messages)``) that writes a kernel, gets the verifier's feedback
  on it and revises it, for ``turns`` turns; every turn's kernel is a
  candidate;
* :func:`frontier_policy`: the same loop driven by an external frontier model
  behind an OpenAI-compatible endpoint, with :class:`FrontierUnavailable`
  raised (never a silent empty answer) when the endpoint cannot be reached,
  so a missing baseline is reported as missing rather than scored as a loss.

Reference parity: kore/eval/policies.py (seed / model policies with
feedback rendering) and opus_policy.py (frontier policy, loud unavailability).
"""
from __future__ import annotations

from typing import Callable, List, Optional

from ..obs import get_logger


class FrontierUnavailable(RuntimeError):
    """The frontier model's endpoint could not produce an answer."""


def seed_policy(task) -> List[str]:
    return [task.seed_src]


def render_feedback(obs) -> str:
    """The verifier's verdict as the policy sees it between turns."""
    from ..policy.format import build_turn_feedback
    return build_turn_feedback(obs)


def model_policy(generate: Callable[[List[dict]], str], *, turns: int = 1, env_factory: Optional[Callable] = None
                 ) -> Callable[[object], List[str]]:
    """``generate(messages) -> response``; with ``env_factory`` and
    ``turns > 1`` the policy sees the verifier's feedback on its previous
    kernel and revises it (the environment's replay cache makes the harness's
    re-evaluation of the same source free)."""
    from ..policy.format import SYSTEM_PROMPT, build_task_prompt, parse_response

    def policy(task) -> List[str]:
        msgs = [{"role": "system", "content": SYSTEM_PROMPT}, {"role": "user", "content": build_task_prompt(task)}]
        out: List[str] = []
        env = env_factory(task) if (env_factory is not None and turns > 1) else None
        for t in range(max(1, turns)):
            resp = generate(msgs)
            src = parse_response(resp)["kernel"]
            msgs.append({"role": "assistant", "content": resp})
            if src:
                out.append(src)
            if env is None or t + 1 >= turns:
                break
            fb = render_feedback(env.step(src)) if src else "No FULL_KERNEL section was found in the answer."
            msgs.append({"role": "user", "content": "Verifier feedback:\n" + fb})
        return out
    return policy


def frontier_policy(client=None, *, url: Optional[str] = None, model: Optional[str] = None, turns: int = 1,
                    env_factory: Optional[Callable] = None) -> Callable[[object], List[str]]:
    """``client``: anything with ``generate(messages)``; else an OpenAI-compatible
    endpoint at ``url`` serving ``model``."""
    log = get_logger("eval.frontier")
    if client is None:
        if not url or not model:
            raise FrontierUnavailable("no frontier client and no endpoint (url, model) given")
        from ..data.teacher import HTTPTeacher
        client = HTTPTeacher(model, base_url=url)

    def gen(messages: List[dict]) -> str:
        try:
            out = client.generate(messages)
        except Exception as e:  # noqa: BLE001 - any transport failure means the baseline is missing
            log.warn("frontier model unavailable", error=f"{type(e).__name__}: {e}")
            raise FrontierUnavailable(f"{type(e).__name__}: {e}") from e
        if not out or not out.strip():
            raise FrontierUnavailable("empty answer from the frontier model")
        return out
    return model_policy(gen, turns=turns, env_factory=env_factory)
