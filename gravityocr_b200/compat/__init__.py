"""Drop-in shims with the reference's operator surface: the in-process ``generate_speculative_natcache`` entry and
the served ``SelfSpecDiffusionWorker`` hooks."""
from .natcache import SelfSpecModel, generate_speculative_natcache
from .sglang_worker import ReqToPagePool, SelfSpecDiffusionWorker

__all__ = ["SelfSpecModel", "generate_speculative_natcache", "ReqToPagePool", "SelfSpecDiffusionWorker"]
