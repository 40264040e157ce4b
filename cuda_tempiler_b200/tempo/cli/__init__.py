"""The tempolator command line (``python -m cuda_tempiler_b200.tempo.cli``)."""
