"""Imports every built-in model builder, task and criterion so that the name registries are complete."""
from .models import builders  # noqa: F401
from .tasks import gpt, harness, pseudo  # noqa: F401
from .criterions import cross_entropy, harness_eval, needle  # noqa: F401
