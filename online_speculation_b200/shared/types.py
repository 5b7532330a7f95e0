"""Model-independent data types."""

TokenSequence = tuple[int, ...]
