"""Minimal stand-in for the three monai names the reference loss imports
(``monai.networks.one_hot``, ``monai.utils.LossReduction``,
``monai.losses.DiceLoss``), written from their documented behaviour. Used only by
``tests/golden/make_golden.py`` to import the reference in a container without
monai; never on the product path."""

__version__ = "shim (monai 1.6.1 behaviour)"
