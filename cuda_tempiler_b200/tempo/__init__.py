"""tempo: the arch-agnostic tempolator pipeline (recognize -> space -> prune -> emit -> build ->
verify -> measure -> ship) restated for this repository, plus its plugins.

The plugin boundary is the ``tempo/arch/1`` contract in ``tempo.plugins.base``; the sm_100a
plugin in ``tempo.plugins.sm100`` imports that contract relatively, so the same directory
dropped into the reference tree as ``tempo/plugins/sm100/`` binds to the reference's own
contract module (reference tempo/plugins/base.py) instead of this one.
"""
