"""Host-side mirrors of the reference's ``utils`` modules used by the quantizer objects."""
