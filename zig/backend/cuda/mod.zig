//! doe_cuda: the CUDA device backend for Doe's Zig runtime, a thin shim over
//! libdoe_cuda.so's C ABI (include/doe_cuda.h).
//!
//! This file belongs at runtime/zig/src/backend/cuda/mod.zig of the doerun/doe
//! tree, beside vulkan/mod.zig, and fills the eleven BackendVTable slots of
//! runtime/zig/src/backend/backend_iface.zig:13-31 the way vulkan/mod.zig:500-512
//! does.  Registration: a `doe_cuda` member of BackendId (backend_ids.zig:3-27),
//! an init_backend arm calling `create` (backend_registry.zig:20-42), and a
//! lane in config/backend-runtime-policy.json.  Link with `-ldoe_cuda` (the
//! library carries the CUDA runtime statically; only the NVIDIA driver is
//! needed at run time).
//!
//! No Zig toolchain exists in the environment this file was written in, so
//! it is not compiled here; every call it makes is exercised through the same
//! C ABI by the Python tests (tests/test_gpu_dispatch.py, tests/test_abi.py).
const std = @import("std");
const backend_iface = @import("../backend_iface.zig");
const runtime_types = @import("../runtime_types.zig");
const model_commands = @import("../../model_commands.zig");
const model_compute_types = @import("../../model_compute_types.zig");

// ---- the C ABI (include/doe_cuda.h) -----------------------------------------
pub const DoeBinding = extern struct {
    binding: u32,
    group: u32,
    handle: u64,
    offset: u64,
    size: u64,
    buffer_type: u32,
    reserved: u32 = 0,
};

pub const DoeExecResult = extern struct {
    status: i32 = 0,
    dispatch_count: u32 = 0,
    setup_ns: u64 = 0,
    encode_ns: u64 = 0,
    submit_wait_ns: u64 = 0,
    gpu_timestamp_ns: u64 = 0,
    gpu_timestamp_attempted: u32 = 0,
    gpu_timestamp_valid: u32 = 0,
};

const Ctx = opaque {};
const DOE_OK: c_int = 0;
const DOE_UNSUPPORTED: c_int = 1;

extern "doe_cuda" fn doe_cuda_open(ordinal: c_int, out: *?*Ctx) c_int;
extern "doe_cuda" fn doe_cuda_close(ctx: *Ctx) c_int;
extern "doe_cuda" fn doe_cuda_last_error(ctx: ?*const Ctx) [*:0]const u8;
extern "doe_cuda" fn doe_cuda_buffer_ensure(ctx: *Ctx, handle: u64, bytes: u64) c_int;
extern "doe_cuda" fn doe_cuda_buffer_write(ctx: *Ctx, handle: u64, offset: u64, data: [*]const u8, size: u64) c_int;
extern "doe_cuda" fn doe_cuda_buffer_read(ctx: *Ctx, handle: u64, offset: u64, dst: [*]u8, size: u64) c_int;
extern "doe_cuda" fn doe_cuda_dispatch(ctx: *Ctx, kernel: [*:0]const u8, entry_point: ?[*:0]const u8, x: u32, y: u32, z: u32, bindings: [*]const DoeBinding, num_bindings: u32, result: *DoeExecResult) c_int;
extern "doe_cuda" fn doe_cuda_flush(ctx: *Ctx, wait_ns: *u64) c_int;
extern "doe_cuda" fn doe_cuda_prewarm_upload(ctx: *Ctx, max_upload_bytes: u64) c_int;
extern "doe_cuda" fn doe_cuda_prewarm_kernel(ctx: *Ctx, kernel: [*:0]const u8) c_int;
extern "doe_cuda" fn doe_cuda_set_upload_behavior(ctx: *Ctx, mode: c_int, submit_every: u32) c_int;
extern "doe_cuda" fn doe_cuda_set_queue_wait_mode(ctx: *Ctx, mode: c_int) c_int;
extern "doe_cuda" fn doe_cuda_set_queue_sync_mode(ctx: *Ctx, per_command: c_int) c_int;
extern "doe_cuda" fn doe_cuda_set_gpu_timestamp_mode(ctx: *Ctx, on: c_int) c_int;

// ---- the backend -------------------------------------------------------------
pub const CudaBackend = struct {
    allocator: std.mem.Allocator,
    ctx: *Ctx,
    // kernel names handed to the C ABI need a terminating zero; dispatches
    // reuse one scratch buffer (the backend is single-threaded per instance)
    name_buf: std.ArrayListUnmanaged(u8) = .{},
    entry_buf: std.ArrayListUnmanaged(u8) = .{},
    bind_buf: std.ArrayListUnmanaged(DoeBinding) = .{},
};

fn cast(ctx: *anyopaque) *CudaBackend {
    return @ptrCast(@alignCast(ctx));
}

fn last_error(self: *CudaBackend) []const u8 {
    return std.mem.span(doe_cuda_last_error(self.ctx));
}

fn z_string(buf: *std.ArrayListUnmanaged(u8), allocator: std.mem.Allocator, s: []const u8) ![*:0]const u8 {
    buf.clearRetainingCapacity();
    try buf.appendSlice(allocator, s);
    try buf.append(allocator, 0);
    return @ptrCast(buf.items.ptr);
}

fn result_of(self: *CudaBackend, rc: c_int, r: DoeExecResult) runtime_types.NativeExecutionResult {
    return .{
        .status = if (rc == DOE_OK) .ok else if (rc == DOE_UNSUPPORTED) .unsupported else .@"error",
        .status_message = if (rc == DOE_OK) "" else last_error(self),
        .setup_ns = r.setup_ns,
        .encode_ns = r.encode_ns,
        .submit_wait_ns = r.submit_wait_ns,
        .dispatch_count = r.dispatch_count,
        .gpu_timestamp_ns = r.gpu_timestamp_ns,
        .gpu_timestamp_attempted = r.gpu_timestamp_attempted != 0,
        .gpu_timestamp_valid = r.gpu_timestamp_valid != 0,
    };
}

/// The init_backend arm (backend_registry.zig:20-42): opens CUDA device
/// `ordinal` and returns the BackendIface.
pub fn create(allocator: std.mem.Allocator, ordinal: c_int) !backend_iface.BackendIface {
    var ctx: ?*Ctx = null;
    if (doe_cuda_open(ordinal, &ctx) != DOE_OK or ctx == null) return error.DoeCudaUnavailable;
    const self = try allocator.create(CudaBackend);
    self.* = .{ .allocator = allocator, .ctx = ctx.? };
    return .{ .id = .doe_cuda, .context = self, .vtable = &VTABLE, .telemetry = .{} };
}

fn deinit(ctx: *anyopaque) void {
    const self = cast(ctx);
    _ = doe_cuda_close(self.ctx);
    self.name_buf.deinit(self.allocator);
    self.entry_buf.deinit(self.allocator);
    self.bind_buf.deinit(self.allocator);
    self.allocator.destroy(self);
}

fn execute_command(ctx: *anyopaque, command: model_commands.Command) anyerror!runtime_types.NativeExecutionResult {
    const self = cast(ctx);
    switch (command) {
        .kernel_dispatch => |kd| {
            const src = kd.bindings orelse &[_]model_compute_types.KernelBinding{};
            self.bind_buf.clearRetainingCapacity();
            for (src) |b| {
                if (b.resource_kind != .buffer)
                    return .{ .status = .unsupported, .status_message = "doe_cuda: only buffer bindings" };
                try self.bind_buf.append(self.allocator, .{
                    .binding = b.binding,
                    .group = b.group,
                    .handle = b.resource_handle,
                    .offset = b.buffer_offset,
                    .size = b.buffer_size,
                    .buffer_type = b.buffer_type,
                });
            }
            const name = try z_string(&self.name_buf, self.allocator, kd.kernel);
            const entry: ?[*:0]const u8 = if (kd.entry_point) |e| try z_string(&self.entry_buf, self.allocator, e) else null;
            var total = DoeExecResult{};
            var n: u32 = 0;
            while (n < @max(kd.repeat, 1)) : (n += 1) {
                var r = DoeExecResult{};
                const rc = doe_cuda_dispatch(self.ctx, name, entry, kd.x, kd.y, kd.z, self.bind_buf.items.ptr, @intCast(self.bind_buf.items.len), &r);
                if (rc != DOE_OK) return result_of(self, rc, r);
                total.setup_ns += r.setup_ns;
                total.encode_ns += r.encode_ns;
                total.submit_wait_ns += r.submit_wait_ns;
                total.gpu_timestamp_ns += r.gpu_timestamp_ns;
                total.dispatch_count += r.dispatch_count;
                total.gpu_timestamp_attempted |= r.gpu_timestamp_attempted;
                total.gpu_timestamp_valid = r.gpu_timestamp_valid;
            }
            return result_of(self, DOE_OK, total);
        },
        .buffer_write => |bw| {
            const bytes = std.mem.sliceAsBytes(bw.data);
            if (bw.buffer_size > 0 and doe_cuda_buffer_ensure(self.ctx, bw.handle, bw.buffer_size) != DOE_OK)
                return result_of(self, 2, .{});
            const rc = doe_cuda_buffer_write(self.ctx, bw.handle, bw.offset, bytes.ptr, bytes.len);
            return result_of(self, rc, .{});
        },
        .barrier => {
            var wait_ns: u64 = 0;
            const rc = doe_cuda_flush(self.ctx, &wait_ns);
            return result_of(self, rc, .{ .submit_wait_ns = wait_ns });
        },
        else => return .{ .status = .unsupported, .status_message = "doe_cuda: command outside the compute path" },
    }
}

fn execute_buffer_write_bytes(ctx: *anyopaque, handle: u64, offset: u64, buffer_size: u64, data: []const u8) anyerror!runtime_types.NativeExecutionResult {
    const self = cast(ctx);
    if (buffer_size > 0 and doe_cuda_buffer_ensure(self.ctx, handle, buffer_size) != DOE_OK)
        return result_of(self, 2, .{});
    return result_of(self, doe_cuda_buffer_write(self.ctx, handle, offset, data.ptr, data.len), .{});
}

fn set_upload_behavior(ctx: *anyopaque, mode: runtime_types.UploadBufferUsageMode, submit_every: u32) void {
    const m: c_int = switch (mode) {
        .copy_dst_copy_src => 0,
        .copy_dst => 1,
    };
    _ = doe_cuda_set_upload_behavior(cast(ctx).ctx, m, submit_every);
}

fn set_queue_wait_mode(ctx: *anyopaque, mode: runtime_types.QueueWaitMode) void {
    const m: c_int = switch (mode) {
        .process_events => 0,
        .wait_any => 1,
    };
    _ = doe_cuda_set_queue_wait_mode(cast(ctx).ctx, m);
}

fn set_queue_sync_mode(ctx: *anyopaque, mode: runtime_types.QueueSyncMode) void {
    _ = doe_cuda_set_queue_sync_mode(cast(ctx).ctx, if (mode == .per_command) 1 else 0);
}

fn set_gpu_timestamp_mode(ctx: *anyopaque, mode: runtime_types.GpuTimestampMode) void {
    _ = doe_cuda_set_gpu_timestamp_mode(cast(ctx).ctx, if (mode == .off) 0 else 1);
}

fn flush_queue(ctx: *anyopaque) anyerror!u64 {
    const self = cast(ctx);
    var wait_ns: u64 = 0;
    if (doe_cuda_flush(self.ctx, &wait_ns) != DOE_OK) return error.DoeCudaFlushFailed;
    return wait_ns;
}

fn prewarm_upload_path(ctx: *anyopaque, max_upload_bytes: u64) anyerror!void {
    if (doe_cuda_prewarm_upload(cast(ctx).ctx, max_upload_bytes) != DOE_OK) return error.DoeCudaPrewarmFailed;
}

fn prewarm_kernel_dispatch(
    ctx: *anyopaque,
    kernel: []const u8,
    entry_point: ?[]const u8,
    bindings: ?[]const model_compute_types.KernelBinding,
    initialize_buffers_on_create: bool,
) anyerror!void {
    _ = entry_point;
    const self = cast(ctx);
    if (initialize_buffers_on_create) {
        // buffers are zero-filled when created; creating them now moves the
        // allocation out of the first timed dispatch
        for (bindings orelse &[_]model_compute_types.KernelBinding{}) |b| {
            if (b.resource_kind == .buffer and b.buffer_size != std.math.maxInt(u64) and b.buffer_size > 0)
                _ = doe_cuda_buffer_ensure(self.ctx, b.resource_handle, b.buffer_offset + b.buffer_size);
        }
    }
    const name = try z_string(&self.name_buf, self.allocator, kernel);
    if (doe_cuda_prewarm_kernel(self.ctx, name) != DOE_OK) return error.DoeCudaKernelUnsupported;
}

fn capture_buffer(ctx: *anyopaque, allocator: std.mem.Allocator, handle: u64, offset: u64, size: u64) anyerror![]u8 {
    const self = cast(ctx);
    const out = try allocator.alloc(u8, size);
    errdefer allocator.free(out);
    if (doe_cuda_buffer_read(self.ctx, handle, offset, out.ptr, size) != DOE_OK) return error.DoeCudaCaptureFailed;
    return out;
}

const VTABLE = backend_iface.BackendVTable{
    .deinit = deinit,
    .execute_command = execute_command,
    .execute_buffer_write_bytes = execute_buffer_write_bytes,
    .set_upload_behavior = set_upload_behavior,
    .set_queue_wait_mode = set_queue_wait_mode,
    .set_queue_sync_mode = set_queue_sync_mode,
    .set_gpu_timestamp_mode = set_gpu_timestamp_mode,
    .flush_queue = flush_queue,
    .prewarm_upload_path = prewarm_upload_path,
    .prewarm_kernel_dispatch = prewarm_kernel_dispatch,
    .capture_buffer = capture_buffer,
};
