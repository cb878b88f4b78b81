from metellus_b200.api.run import RunResult, run

__all__ = ["RunResult", "run"]
