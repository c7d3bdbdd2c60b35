"""Per-request sampling parameters.

Parity: ``nanovllm/sampling_params.py:4-11`` (temperature >= 0, max_tokens,
ignore_eos).  ``temperature <= 1e-10`` means greedy.
"""

from dataclasses import dataclass


@dataclass(slots=True)
class SamplingParams:
    temperature: float = 1.0
    max_tokens: int = 64
    ignore_eos: bool = False

    def __post_init__(self):
        if self.temperature < 0:
            raise ValueError("temperature must be non-negative")
        if self.max_tokens <= 0:
            raise ValueError("max_tokens must be positive")

    @property
    def is_greedy(self) -> bool:
        return self.temperature <= 1e-10
