// Error plumbing shared by the C ABI translation units.
#pragma once
#include <string>

void db_set_error(const char* code, const std::string& message);
int db_fail(int status, const char* code, const std::string& message);
int db_cuda_status(int cuda_error, const char* what);
int* db_device_error_ptr();
