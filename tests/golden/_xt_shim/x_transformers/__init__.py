"""Test-only stand-in for the ``x_transformers`` package (pinned 2.23.5 by the
reference, not installed in this container).  Only the two names the reference
DiT imports are provided; see ``x_transformers.py`` in this folder."""
