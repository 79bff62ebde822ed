"""Device availability (reference ``runtime/utils.py:3-19``)."""


def is_b200_compatible() -> bool:
    """True when libnkb loads and at least one sm_100 device is visible."""
    try:
        from nkipy_b200.spike.runtime import Spike

        n = Spike.get_visible_neuron_core_count()
    except Exception as e:  # noqa: BLE001
        print(f"Device compatibility check failed: {e}")
        return False
    if n < 1:
        print("No CUDA devices found")
        return False
    return True


# reference-compatible name
is_neuron_compatible = is_b200_compatible
