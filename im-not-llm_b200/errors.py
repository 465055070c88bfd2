"""The error type of the engine API, mirroring the reference's InlError
(crates/inl-core/src/error.rs:5-46): one class per variant and the same stable
``code`` strings (``InlError::code``, :36-46)."""
from __future__ import annotations


class InlError(Exception):
    code = "other"

    def __init__(self, message: str):
        super().__init__(message)
        self.message = message

    def __str__(self) -> str:  # same prefixes as the reference's #[error] texts
        prefix = {
            "config": "config error: ",
            "inference": "inference failed: ",
            "timeout": "inference timeout: ",
            "invalid_input": "invalid input: ",
        }.get(self.code, "")
        return prefix + self.message

    @staticmethod
    def config(msg: str) -> "ConfigError":
        return ConfigError(msg)

    @staticmethod
    def inference(msg: str) -> "InferenceError":
        return InferenceError(msg)

    @staticmethod
    def timeout(msg: str) -> "TimeoutError_":
        return TimeoutError_(msg)

    @staticmethod
    def invalid_input(msg: str) -> "InvalidInputError":
        return InvalidInputError(msg)


class ConfigError(InlError):
    code = "config"


class InferenceError(InlError):
    code = "inference"


class TimeoutError_(InlError):
    code = "timeout"


class InvalidInputError(InlError):
    code = "invalid_input"


# INL_ERR_* status codes of include/inl_cuda.h.
_STATUS = {1: ConfigError, 2: InferenceError, 3: TimeoutError_, 4: InvalidInputError}


def error_for_status(status: int, message: str) -> InlError:
    return _STATUS.get(status, InlError)(message)
