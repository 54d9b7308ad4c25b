"""air_rs.utils."""
