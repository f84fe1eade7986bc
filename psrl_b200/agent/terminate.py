"""Why a rollout trajectory stopped, and what recovery each reason calls for.

The classification follows the reference's ``TerminateReason``
(``psrl/workers/agent_loop/loops/utils.py:34-80``):

* successful (usable training data): finished, length / turn limits;
* worker retry (try the trajectory again, up to ``rollout.agent.retry_limit``
  attempts): timeouts (environment or whole trajectory) and errors;
* manager retry (the group's buffer slot is lost, so the manager aborts the
  group and dispatches a fresh prompt): errors and trajectory timeouts that
  are still failing after the last attempt;
* aborted: stopped on purpose by the staleness protocol; no recovery.
"""

from __future__ import annotations

from enum import Enum


class TerminateReason(Enum):
    FINISHED = "finished"
    MAX_RESPONSE_LENGTH_EXCEEDED = "max_response_length_exceeded"
    MAX_TURNS_EXCEEDED = "max_turns_exceeded"
    ENV_TIMEOUT = "env_timeout"
    TRAJECTORY_TIMEOUT = "trajectory_timeout"
    ABORTED = "aborted"
    UNKNOWN = "unknown"
    ROLLOUT_ERROR = "rollout_error"

    @property
    def is_successful(self) -> bool:
        return self in (TerminateReason.FINISHED, TerminateReason.MAX_TURNS_EXCEEDED,
                        TerminateReason.MAX_RESPONSE_LENGTH_EXCEEDED)

    @property
    def is_timeout(self) -> bool:
        return self in (TerminateReason.ENV_TIMEOUT, TerminateReason.TRAJECTORY_TIMEOUT)

    @property
    def is_error(self) -> bool:
        return self in (TerminateReason.ROLLOUT_ERROR, TerminateReason.UNKNOWN)

    @property
    def is_aborted(self) -> bool:
        return self is TerminateReason.ABORTED

    def needs_worker_retry(self) -> bool:
        return self.is_timeout or self.is_error

    def needs_manager_retry(self) -> bool:
        return self.is_error or self is TerminateReason.TRAJECTORY_TIMEOUT


def reason_of_exception(exc: BaseException) -> TerminateReason:
    """An environment step that timed out is ENV_TIMEOUT; anything else raised
    while finishing a trajectory (environment, tool, reward) is ROLLOUT_ERROR."""
    if isinstance(exc, TimeoutError):
        return TerminateReason.ENV_TIMEOUT
    return TerminateReason.ROLLOUT_ERROR


def reason_of_finish(finish_reason: str | None) -> TerminateReason:
    """Map an engine ``RequestOutput.finish_reason`` onto a reason."""
    return {
        "stop": TerminateReason.FINISHED,
        "length": TerminateReason.MAX_RESPONSE_LENGTH_EXCEEDED,
        "abort": TerminateReason.ABORTED,
        "timeout": TerminateReason.TRAJECTORY_TIMEOUT,
        "error": TerminateReason.ROLLOUT_ERROR,
    }.get(finish_reason or "", TerminateReason.UNKNOWN)
