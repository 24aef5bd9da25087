"""Host-side mirror of clj-xla for the decoder path (tracer, printer, models,
drivers, PJRT ctypes bindings)."""
